// kq_accept.cuh -- on-device acceptance of a verified draft tree and K/V compaction (sm_100a).
//
// k_accept implements, bit for bit, the deterministic speculative-sampling rule of the CPU
// oracle (or_accept): at node v with target p_v = softmax(z_v / T) and draft q_v = softmax(g_v),
// children c in increasing id are accepted iff u_acc[c] * q(d_c) < p(d_c); a rejection replaces p
// by the normalised residual max(0, p - q) (p_v again if the residual is empty); when no child is
// accepted the token is the inverse-CDF sample of p at u_fin[v]. T = 0 is greedy matching against
// the argmax (lowest id on ties). It generalises the reference's one-hot-draft chain acceptance
// (scripts/kindi_q4/kindi/spec.py:769-787) to draft distributions and trees.
//
// Exactness: one CTA of 1024 threads. e^t is kq_exp (Cody-Waite reduction, Taylor degree 7, the
// same fp32 operations as the oracle); vocabulary sums are blocked exactly as in the oracle:
// blocks of 1024 consecutive ids, thread i holding id b*1024 + i, each block summed by the
// xor-shuffle tree over lanes and then over warps (a balanced pairwise tree over the block), the
// block sums added in order by one thread; the inverse CDF is sequential in one thread. Divisions
// are correctly rounded (__fdiv_rn), products and sums unfused.
//
// k_commit moves the K/V rows of the accepted path to consecutive positions: the accepted node
// path[j] (j >= 1) leaves slot pos + path[j] for position pos + j, in increasing j.
#pragma once
#include "kq_common.cuh"
#include <cfloat>

namespace kq {

constexpr int ACC_THREADS = 1024, ACC_BLK = 1024, ACC_MAX_BLOCKS = 256;   // vocabularies up to 262144
#ifndef KQ_MAX_TREE
#define KQ_MAX_TREE 128   // draft-tree nodes (include/kq.h)
#endif

__device__ __forceinline__ float kq_exp(float t) {
  if (!(t >= -87.0f)) return 0.0f;
  const float k = __fsub_rn(__fmaf_rn(t, 0x1.715476p+0f, 12582912.0f), 12582912.0f);   // round(t / ln2)
  float r = __fmaf_rn(-k, 0x1.62e4p-1f, t);
  r = __fmaf_rn(-k, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;                // 1/5040
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);     // 1/720
  p = __fmaf_rn(p, r, 0x1.111112p-7f);      // 1/120
  p = __fmaf_rn(p, r, 0x1.555556p-5f);      // 1/24
  p = __fmaf_rn(p, r, 0x1.555556p-3f);      // 1/6
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  return __fmul_rn(p, __int_as_float(((int)k + 127) << 23));
}

struct AcceptParams {
  const float* z;        // target logits [n][V] (the verify pass)
  const float* g;        // draft logits [n][V] (row v: the distribution of v's children)
  const int* tokens;     // [n]
  const int* parents;    // [n], parents[0] = -1
  const float* u_acc;    // [n]
  const float* u_fin;    // [n]
  int n, V;
  float tau;             // 1/T as fp32; 0 = greedy
  float* p;              // [V] scratch
  float* q;              // [V] scratch
  int* path;             // out: [n + 1] accepted nodes (path[0] = 0)
  int* out;              // out: [n + 1] emitted tokens
  int* count;            // out: [2] emitted tokens, path length
};

struct AccShared {
  float bs[ACC_MAX_BLOCKS];
  float wsum[32];
  float fval[32];
  int fidx[32];
  float S;
  int pick;
};

// Block sums of w (thread i owns ids b*1024 + i) into sh.bs, their in-order total returned to all.
__device__ float acc_blocked_sum(const float* w, int V, AccShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (V + ACC_BLK - 1) / ACC_BLK;
  for (int b = 0; b < nb; ++b) {
    const int id = b * ACC_BLK + tid;
    float v = id < V ? w[id] : 0.0f;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) sh.wsum[warp] = v;
    __syncthreads();
    if (warp == 0) {
      float t = sh.wsum[lane];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
      if (lane == 0) sh.bs[b] = t;
    }
    __syncthreads();
  }
  if (tid == 0) {
    float tot = 0.0f;
    for (int b = 0; b < nb; ++b) tot = __fadd_rn(tot, sh.bs[b]);
    sh.S = tot;
  }
  __syncthreads();
  return sh.S;
}

// Largest value of z (and its lowest index) over the CTA.
__device__ void acc_argmax(const float* z, int V, AccShared& sh, float& best, int& bidx) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float v = -INFINITY;
  int vi = 0x7fffffff;
  for (int i = tid; i < V; i += ACC_THREADS) {
    const float x = z[i];
    if (x > v || (x == v && i < vi)) { v = x; vi = i; }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, off);
    const int oi = __shfl_xor_sync(0xffffffffu, vi, off);
    if (ov > v || (ov == v && oi < vi)) { v = ov; vi = oi; }
  }
  if (lane == 0) { sh.fval[warp] = v; sh.fidx[warp] = vi; }
  __syncthreads();
  if (tid == 0) {
    float bv = sh.fval[0];
    int bi = sh.fidx[0];
    for (int w = 1; w < 32; ++w)
      if (sh.fval[w] > bv || (sh.fval[w] == bv && sh.fidx[w] < bi)) { bv = sh.fval[w]; bi = sh.fidx[w]; }
    sh.fval[0] = bv;
    sh.fidx[0] = bi;
  }
  __syncthreads();
  best = sh.fval[0];
  bidx = sh.fidx[0] == 0x7fffffff ? 0 : sh.fidx[0];
  __syncthreads();
}

// p = softmax(z * tau): max, kq_exp, blocked sum, correctly rounded division.
__device__ void acc_softmax(const float* z, int V, float tau, float* p, AccShared& sh) {
  float mx;
  int mi;
  acc_argmax(z, V, sh, mx, mi);
  for (int i = threadIdx.x; i < V; i += ACC_THREADS) p[i] = kq_exp(__fmul_rn(__fsub_rn(z[i], mx), tau));
  __syncthreads();
  const float S = acc_blocked_sum(p, V, sh);
  for (int i = threadIdx.x; i < V; i += ACC_THREADS) p[i] = __fdiv_rn(p[i], S);
  __syncthreads();
}

__global__ void __launch_bounds__(ACC_THREADS, 1) k_accept(const AcceptParams A) {
  __shared__ AccShared sh;
  const int tid = threadIdx.x, V = A.V, n = A.n;
  int v = 0, np = 0, no = 0;
  if (tid == 0) A.path[np] = 0;
  ++np;
  for (int guard = 0; guard <= n; ++guard) {
    const float* zv = A.z + (size_t)v * V;
    int acc = -1;
    if (A.tau == 0.0f) {
      float bv;
      int best;
      acc_argmax(zv, V, sh, bv, best);
      for (int c = v + 1; c < n && acc < 0; ++c)
        if (A.parents[c] == v && A.tokens[c] == best) acc = c;
      if (acc < 0) {
        if (tid == 0) A.out[no] = best;
        ++no;
        break;
      }
    } else {
      acc_softmax(zv, V, A.tau, A.p, sh);
      bool first = true;
      for (int c = v + 1; c < n && acc < 0; ++c) {
        if (A.parents[c] != v) continue;
        if (first) { acc_softmax(A.g + (size_t)v * V, V, 1.0f, A.q, sh); first = false; }
        const int d = A.tokens[c];
        if (__fmul_rn(A.u_acc[c], A.q[d]) < A.p[d]) { acc = c; break; }
        for (int i = tid; i < V; i += ACC_THREADS) {
          const float r = __fsub_rn(A.p[i], A.q[i]);
          A.p[i] = r > 0.0f ? r : 0.0f;
        }
        __syncthreads();
        const float R = acc_blocked_sum(A.p, V, sh);
        if (R > 0.0f) {
          for (int i = tid; i < V; i += ACC_THREADS) A.p[i] = __fdiv_rn(A.p[i], R);
          __syncthreads();
        } else {
          acc_softmax(zv, V, A.tau, A.p, sh);   // empty residual (p == q): back to p_v
        }
      }
      if (acc < 0) {
        // inverse CDF of p at u_fin[v]
        const float W = acc_blocked_sum(A.p, V, sh);
        if (tid == 0) {
          const float target = __fmul_rn(A.u_fin[v], W);
          const int nb = (V + ACC_BLK - 1) / ACC_BLK;
          float prefix = 0.0f;
          int pick = -1;
          for (int b = 0; b < nb && pick < 0; ++b) {
            if (__fadd_rn(prefix, sh.bs[b]) > target) {
              float run = prefix;
              for (int i = b * ACC_BLK; i < V && i < (b + 1) * ACC_BLK; ++i) {
                run = __fadd_rn(run, A.p[i]);
                if (run > target) { pick = i; break; }
              }
            }
            prefix = __fadd_rn(prefix, sh.bs[b]);
          }
          sh.pick = pick;
        }
        __syncthreads();
        if (sh.pick < 0) {
          // rounding left the target above every running sum: the largest id with p > 0 (0 if
          // none), as a block-wide max instead of one thread scanning down the vocabulary
          int hi = -1;
          for (int i = tid; i < V; i += ACC_THREADS)
            if (A.p[i] > 0.0f) hi = i;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, off));
          if ((tid & 31) == 0) sh.fidx[tid >> 5] = hi;
          __syncthreads();
          if (tid == 0) {
            int b = -1;
            for (int w = 0; w < ACC_THREADS / 32; ++w) b = max(b, sh.fidx[w]);
            sh.pick = b < 0 ? 0 : b;
          }
          __syncthreads();
        }
        if (tid == 0) A.out[no] = sh.pick;
        __syncthreads();
        ++no;
        break;
      }
    }
    if (tid == 0) {
      A.out[no] = A.tokens[acc];
      A.path[np] = acc;
    }
    ++no;
    ++np;
    v = acc;
  }
  if (tid == 0) {
    A.count[0] = no;
    A.count[1] = np;
  }
}

// K/V compaction, one CTA per (layer, K or V): rows of the accepted nodes to consecutive
// positions, in increasing j. Cache layout [n_kv][ctx][hd] per layer and tensor.
struct CommitParams {
  __half* const* caches;   // [2 * n_layers]: K of layer l at 2l, V at 2l + 1
  const int* path;         // [k + 1], path[0] = 0
  int k, pos, n_kv, ctx, hd;
};
__global__ void k_commit(const CommitParams C) {
  __half* cache = C.caches[blockIdx.x];
  for (int j = 1; j <= C.k; ++j) {
    const int src = C.pos + C.path[j], dst = C.pos + j;
    if (src != dst)
      for (int e = threadIdx.x; e < C.n_kv * C.hd; e += blockDim.x) {
        const int kv = e / C.hd, d = e % C.hd;
        cache[((size_t)kv * C.ctx + dst) * C.hd + d] = cache[((size_t)kv * C.ctx + src) * C.hd + d];
      }
    __syncthreads();
  }
}

}  // namespace kq
