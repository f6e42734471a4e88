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
// blocks of 1024 consecutive ids, each block summed as a balanced pairwise tree (over the 32 ids
// of a row, then over the 32 rows; acc_blocked_sum says how one warp forms it), the block sums
// added in order by one thread; the inverse CDF is sequential in one thread. Divisions
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
  float blk[ACC_BLK];   // the block the inverse CDF scans
  float S, prefix;
  int pick, cand;
};

// Block sums of w into sh.bs, their in-order total returned to all. The sum of block b is defined
// as the one-block-per-pass form computes it: thread i = 32 r + l holds id b*1024 + i, each row r
// of 32 ids is summed by the xor-shuffle tree over lanes (lane bit 0 paired first), then the 32
// row sums by the same tree over rows. Here one warp sums a whole block on its own: lane l loads
// column l of all 32 rows, a reduce-scatter butterfly over the lanes (step k adds the partial sums
// of the lanes differing in bit k, each lane keeping half of the rows: the rows whose top
// remaining bit equals bit k of the lane) leaves in lane l the full lane tree of row
// bitreverse(l), and the xor tree over the lanes from bit 4 down to bit 0 then pairs the rows
// from row bit 0 up. Every addition pairs the same two partial sums as the per-row trees (fp32
// addition is commutative), so the block sums are bit-identical to that form; the warps work on
// different blocks at once and the CTA meets at one barrier instead of two per block.
__device__ float acc_blocked_sum(const float* w, int V, AccShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = (V + ACC_BLK - 1) / ACC_BLK;
  for (int b = warp; b < nb; b += ACC_THREADS / 32) {
    float x[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      const int id = b * ACC_BLK + r * 32 + lane;
      x[r] = id < V ? w[id] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const int m = 16 >> k;                       // rows kept after this step
      const bool keep_hi = (lane >> k) & 1;
#pragma unroll
      for (int i = 0; i < m; ++i) {
        const float send = keep_hi ? x[i] : x[i + m];
        const float kept = keep_hi ? x[i + m] : x[i];
        x[i] = __fadd_rn(kept, __shfl_xor_sync(0xffffffffu, send, 1 << k));
      }
    }
    float t = x[0];                                // lane tree of row bitreverse(lane)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
    if (lane == 0) sh.bs[b] = t;
  }
  __syncthreads();
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
  // elementwise passes read 4 ids per thread per step when V is a multiple of 4 (rows then start
  // on 16 bytes): one CTA needs many loads in flight to stream from L2; the result does not
  // depend on which thread sees which id
  const int V4 = (V & 3) ? 0 : V;
#pragma unroll 4
  for (int i = 4 * tid; i < V4; i += 4 * ACC_THREADS) {
    const float4 x = *reinterpret_cast<const float4*>(z + i);
    if (x.x > v || (x.x == v && i < vi)) { v = x.x; vi = i; }
    if (x.y > v || (x.y == v && i + 1 < vi)) { v = x.y; vi = i + 1; }
    if (x.z > v || (x.z == v && i + 2 < vi)) { v = x.z; vi = i + 2; }
    if (x.w > v || (x.w == v && i + 3 < vi)) { v = x.w; vi = i + 3; }
  }
#pragma unroll 8
  for (int i = V4 + tid; i < V; i += ACC_THREADS) {
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

// p[i] = p[i] / S, correctly rounded, for every id; ends with a CTA barrier.
__device__ void acc_scale(float* p, int V, float S) {
  const int V4 = (V & 3) ? 0 : V;
#pragma unroll 4
  for (int i = 4 * threadIdx.x; i < V4; i += 4 * ACC_THREADS) {
    const float4 x = *reinterpret_cast<const float4*>(p + i);
    *reinterpret_cast<float4*>(p + i) = make_float4(__fdiv_rn(x.x, S), __fdiv_rn(x.y, S), __fdiv_rn(x.z, S), __fdiv_rn(x.w, S));
  }
  for (int i = V4 + threadIdx.x; i < V; i += ACC_THREADS) p[i] = __fdiv_rn(p[i], S);
  __syncthreads();
}

// p = softmax(z * tau): max, kq_exp, blocked sum, correctly rounded division.
__device__ void acc_softmax(const float* z, int V, float tau, float* p, AccShared& sh) {
  float mx;
  int mi;
  acc_argmax(z, V, sh, mx, mi);
  const int V4 = (V & 3) ? 0 : V;
#pragma unroll 4
  for (int i = 4 * threadIdx.x; i < V4; i += 4 * ACC_THREADS) {
    const float4 x = *reinterpret_cast<const float4*>(z + i);
    *reinterpret_cast<float4*>(p + i) = make_float4(kq_exp(__fmul_rn(__fsub_rn(x.x, mx), tau)), kq_exp(__fmul_rn(__fsub_rn(x.y, mx), tau)),
                                                    kq_exp(__fmul_rn(__fsub_rn(x.z, mx), tau)), kq_exp(__fmul_rn(__fsub_rn(x.w, mx), tau)));
  }
  for (int i = V4 + threadIdx.x; i < V; i += ACC_THREADS) p[i] = kq_exp(__fmul_rn(__fsub_rn(z[i], mx), tau));
  __syncthreads();
  const float S = acc_blocked_sum(p, V, sh);
  acc_scale(p, V, S);
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
        const int V4 = (V & 3) ? 0 : V;
#pragma unroll 4
        for (int i = 4 * tid; i < V4; i += 4 * ACC_THREADS) {
          const float4 pp = *reinterpret_cast<const float4*>(A.p + i), qq = *reinterpret_cast<const float4*>(A.q + i);
          const float r0 = __fsub_rn(pp.x, qq.x), r1 = __fsub_rn(pp.y, qq.y), r2 = __fsub_rn(pp.z, qq.z), r3 = __fsub_rn(pp.w, qq.w);
          *reinterpret_cast<float4*>(A.p + i) = make_float4(r0 > 0.0f ? r0 : 0.0f, r1 > 0.0f ? r1 : 0.0f, r2 > 0.0f ? r2 : 0.0f, r3 > 0.0f ? r3 : 0.0f);
        }
        for (int i = V4 + tid; i < V; i += ACC_THREADS) {
          const float r = __fsub_rn(A.p[i], A.q[i]);
          A.p[i] = r > 0.0f ? r : 0.0f;
        }
        __syncthreads();
        const float R = acc_blocked_sum(A.p, V, sh);
        if (R > 0.0f) {
          acc_scale(A.p, V, R);
        } else {
          acc_softmax(zv, V, A.tau, A.p, sh);   // empty residual (p == q): back to p_v
        }
      }
      if (acc < 0) {
        // inverse CDF of p at u_fin[v]: the blocks in order, prefix = the in-order sum of the block
        // sums before block b; a block whose prefix + sum exceeds the target is scanned id by id
        // from the prefix (rounding can leave the target above every running sum of it: then the
        // walk goes on with the next blocks). The candidate block is first staged in shared memory
        // by all threads, and one thread scans it there.
        const float W = acc_blocked_sum(A.p, V, sh);
        const float target = __fmul_rn(A.u_fin[v], W);
        const int nb = (V + ACC_BLK - 1) / ACC_BLK;
        if (tid == 0) { sh.prefix = 0.0f; sh.cand = 0; sh.pick = -1; }
        __syncthreads();
        for (;;) {
          if (tid == 0) {   // the next candidate block from sh.cand on
            float prefix = sh.prefix;
            int b = sh.cand;
            while (b < nb && !(__fadd_rn(prefix, sh.bs[b]) > target)) { prefix = __fadd_rn(prefix, sh.bs[b]); ++b; }
            sh.prefix = prefix;
            sh.cand = b;
          }
          __syncthreads();
          const int b = sh.cand;
          if (b >= nb) break;
          const int id = b * ACC_BLK + tid;
          sh.blk[tid] = id < V ? A.p[id] : 0.0f;
          __syncthreads();
          if (tid == 0) {
            float run = sh.prefix;
            for (int i = b * ACC_BLK; i < V && i < (b + 1) * ACC_BLK; ++i) {
              run = __fadd_rn(run, sh.blk[i - b * ACC_BLK]);
              if (run > target) { sh.pick = i; break; }
            }
            sh.prefix = __fadd_rn(sh.prefix, sh.bs[b]);
            sh.cand = b + 1;
          }
          __syncthreads();
          if (sh.pick >= 0) break;
        }
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
