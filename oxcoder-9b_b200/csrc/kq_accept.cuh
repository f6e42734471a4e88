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
// Exactness (k_accept: one CTA of 1024 threads; k_accept_grid below: the same arithmetic over a
// cooperative grid). e^t is kq_exp (Cody-Waite reduction, Taylor degree 7, the
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
#include <cstddef>

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
  int* err;              // device error word (the multi-CTA form's grid-barrier waits)
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

// ------------------------------------------------------------------------------ multi-CTA form
// The same rule with the same arithmetic over a cooperative grid: CTA c owns the 1024-id blocks c
// and c + gridDim.x (gridDim.x = ceil(blocks / 2)), one id per thread per block, and keeps its p
// and q values in registers. Everything elementwise stays in the CTA; a vocabulary-wide result
// (the argmax, a blocked sum, an acceptance decision, the inverse-CDF pick) goes through global
// memory and a software grid barrier, after which every CTA forms it the same way: the block sums
// are each formed by one warp exactly as acc_blocked_sum forms them and added in block order by
// one thread of every CTA; the argmax keeps the lowest id among equal values; the inverse CDF
// takes, of the blocks whose in-order prefix plus sum exceeds the target, the first whose
// one-thread scan finds the id. So every result is bit-identical to k_accept's. The exchange
// arrays alternate between two halves by barrier parity: a CTA that runs ahead writes the half
// that no other CTA can still be reading. Barrier waits are bounded (KQ_DEV_ERR_GRID).
constexpr uint32_t ACC_GRID_WAIT_LIMIT = 1u << 22;   // acquire polls (~seconds) before giving up
struct AccGridScratch {
  unsigned bar;          // barrier arrivals (cleared by the host before each launch)
  unsigned pick;         // inverse-CDF pick: the smallest found id (host: 0xFFFFFFFF)
  int hi;                // fallback: the largest id with p > 0 (host: -1)
  int decision[2];       // acceptance decision of the current child, by barrier parity
  float bs[2][ACC_MAX_BLOCKS];
  float val[2][ACC_MAX_BLOCKS];
  int idx[2][ACC_MAX_BLOCKS];
};
static_assert(offsetof(AccGridScratch, hi) == offsetof(AccGridScratch, pick) + sizeof(unsigned),
              "pick and hi are cleared by one host memset");
struct AccGridShared {
  float blk[2][ACC_BLK];   // this CTA's blocks of the last blocked sum
  float sbs[ACC_MAX_BLOCKS];   // the grid's block sums / per-CTA maxima, staged by all threads at
  float sval[ACC_MAX_BLOCKS];  // once (one L2 round trip) before one thread combines them in order
  int sidx[ACC_MAX_BLOCKS];
  float wval[32];
  int widx[32];
  float S, bv;
  int bi, fail;
};
__device__ __forceinline__ unsigned acc_ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Grid barrier number gen (1, 2, ...); false when this CTA's wait gave up (or another CTA's did).
__device__ bool acc_grid_sync(AccGridScratch* G, unsigned gen, int* err, AccGridShared& sh) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(&G->bar, 1u);
    const unsigned target = gen * gridDim.x;
    for (uint32_t it = 0; acc_ld_acquire(&G->bar) < target; ++it) {
      if (it > ACC_GRID_WAIT_LIMIT || ((it & 1023) == 1023 && (*(volatile int*)err & KQ_DEV_ERR_GRID))) {
        atomicOr(err, KQ_DEV_ERR_GRID);
        sh.fail = 1;
        break;
      }
    }
  }
  __syncthreads();
  return !sh.fail;
}

__global__ void __launch_bounds__(ACC_THREADS, 1) k_accept_grid(const AcceptParams A, AccGridScratch* G) {
  __shared__ AccGridShared sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, V = A.V, n = A.n;
  const int nb = (V + ACC_BLK - 1) / ACC_BLK, NC = gridDim.x, cta = blockIdx.x;
  const int nown = cta + NC < nb ? 2 : 1;   // this CTA's blocks: cta, cta + NC
  if (tid == 0) sh.fail = 0;
  __syncthreads();
  unsigned gen = 0;
  int idk[2];
#pragma unroll
  for (int kb = 0; kb < 2; ++kb) idk[kb] = kb < nown ? (cta + kb * NC) * ACC_BLK + tid : V;   // V: no id

  // the argmax of a row over the vocabulary (lowest id among equal values), to every thread
  auto argmax = [&](const float* row, float& best, int& bidx) -> bool {
    float v = -INFINITY;
    int vi = 0x7fffffff;
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
      if (idk[kb] < V) {
        const float x = row[idk[kb]];
        if (x > v || (x == v && idk[kb] < vi)) { v = x; vi = idk[kb]; }
      }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, off);
      const int oi = __shfl_xor_sync(0xffffffffu, vi, off);
      if (ov > v || (ov == v && oi < vi)) { v = ov; vi = oi; }
    }
    if (lane == 0) { sh.wval[warp] = v; sh.widx[warp] = vi; }
    __syncthreads();
    const int par = (gen + 1) & 1;
    if (tid == 0) {
      float bv = sh.wval[0];
      int bi = sh.widx[0];
      for (int w = 1; w < 32; ++w)
        if (sh.wval[w] > bv || (sh.wval[w] == bv && sh.widx[w] < bi)) { bv = sh.wval[w]; bi = sh.widx[w]; }
      G->val[par][cta] = bv;
      G->idx[par][cta] = bi;
    }
    if (!acc_grid_sync(G, ++gen, A.err, sh)) return false;
    for (int c = tid; c < NC; c += ACC_THREADS) {
      sh.sval[c] = __ldcg(&G->val[par][c]);
      sh.sidx[c] = __ldcg(&G->idx[par][c]);
    }
    __syncthreads();
    if (tid == 0) {
      float bv = sh.sval[0];
      int bi = sh.sidx[0];
      for (int c = 1; c < NC; ++c) {
        const float cv = sh.sval[c];
        const int ci = sh.sidx[c];
        if (cv > bv || (cv == bv && ci < bi)) { bv = cv; bi = ci; }
      }
      sh.bv = bv;
      sh.bi = bi;
    }
    __syncthreads();
    best = sh.bv;
    bidx = sh.bi == 0x7fffffff ? 0 : sh.bi;
    __syncthreads();
    return true;
  };
  // the in-order total of the block sums of w (acc_blocked_sum's form); sh.blk keeps this CTA's
  // blocks and sh.sbs all block sums until the next call
  auto blocksum = [&](const float (&w)[2], float& S) -> bool {
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
      if (kb < nown) sh.blk[kb][tid] = idk[kb] < V ? w[kb] : 0.0f;
    __syncthreads();
    const int par = (gen + 1) & 1;
    if (warp < nown) {
      float x[32];
#pragma unroll
      for (int r = 0; r < 32; ++r) x[r] = sh.blk[warp][r * 32 + lane];
#pragma unroll
      for (int k = 0; k < 5; ++k) {
        const int m = 16 >> k;
        const bool keep_hi = (lane >> k) & 1;
#pragma unroll
        for (int i = 0; i < m; ++i) {
          const float send = keep_hi ? x[i] : x[i + m];
          const float kept = keep_hi ? x[i + m] : x[i];
          x[i] = __fadd_rn(kept, __shfl_xor_sync(0xffffffffu, send, 1 << k));
        }
      }
      float t = x[0];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
      if (lane == 0) G->bs[par][cta + warp * NC] = t;
    }
    if (!acc_grid_sync(G, ++gen, A.err, sh)) return false;
    for (int b = tid; b < nb; b += ACC_THREADS) sh.sbs[b] = __ldcg(&G->bs[par][b]);
    __syncthreads();
    if (tid == 0) {
      float tot = 0.0f;
      for (int b = 0; b < nb; ++b) tot = __fadd_rn(tot, sh.sbs[b]);
      sh.S = tot;
    }
    __syncthreads();
    S = sh.S;
    __syncthreads();
    return true;
  };
  // p = softmax(row * tau) on this CTA's ids
  auto softmax = [&](const float* row, float tau, float (&p)[2]) -> bool {
    float mx;
    int mi;
    if (!argmax(row, mx, mi)) return false;
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) p[kb] = idk[kb] < V ? kq_exp(__fmul_rn(__fsub_rn(row[idk[kb]], mx), tau)) : 0.0f;
    float S;
    if (!blocksum(p, S)) return false;
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
      if (idk[kb] < V) p[kb] = __fdiv_rn(p[kb], S);
    return true;
  };

  float pv[2] = {0.0f, 0.0f}, qv[2] = {0.0f, 0.0f};
  const bool writer = cta == 0 && tid == 0;
  int v = 0, np = 0, no = 0;
  if (writer) A.path[np] = 0;
  ++np;
  bool ok = true;
  for (int guard = 0; guard <= n && ok; ++guard) {
    const float* zv = A.z + (size_t)v * V;
    int acc = -1;
    if (A.tau == 0.0f) {
      float bv;
      int best;
      if (!(ok = argmax(zv, bv, best))) break;
      for (int c = v + 1; c < n && acc < 0; ++c)
        if (A.parents[c] == v && A.tokens[c] == best) acc = c;
      if (acc < 0) {
        if (writer) A.out[no] = best;
        ++no;
        break;
      }
    } else {
      if (!(ok = softmax(zv, A.tau, pv))) break;
      bool first = true;
      for (int c = v + 1; c < n && acc < 0; ++c) {
        if (A.parents[c] != v) continue;
        if (first) {
          if (!(ok = softmax(A.g + (size_t)v * V, 1.0f, qv))) break;
          first = false;
        }
        // the owner of id d decides, the grid reads its decision
        const int d = A.tokens[c], bd = d / ACC_BLK, par = (gen + 1) & 1;
        if (bd % NC == cta && tid == d % ACC_BLK) {
          const int kb = bd / NC;
          G->decision[par] = __fmul_rn(A.u_acc[c], qv[kb]) < pv[kb] ? 1 : 0;
        }
        if (!(ok = acc_grid_sync(G, ++gen, A.err, sh))) break;
        if (__ldcg(&G->decision[par])) { acc = c; break; }
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
          if (idk[kb] < V) {
            const float r = __fsub_rn(pv[kb], qv[kb]);
            pv[kb] = r > 0.0f ? r : 0.0f;
          }
        float R;
        if (!(ok = blocksum(pv, R))) break;
        if (R > 0.0f) {
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
            if (idk[kb] < V) pv[kb] = __fdiv_rn(pv[kb], R);
        } else if (!(ok = softmax(zv, A.tau, pv))) {   // empty residual (p == q): back to p_v
          break;
        }
      }
      if (!ok) break;
      if (acc < 0) {
        // inverse CDF of p at u_fin[v]: the first block (in order) whose prefix + sum exceeds the
        // target and whose scan from the prefix finds the id; none: the largest id with p > 0
        float W;
        if (!(ok = blocksum(pv, W))) break;
        const float target = __fmul_rn(A.u_fin[v], W);
        if (tid == 0) {
          for (int kb = 0; kb < nown; ++kb) {
            const int b = cta + kb * NC;
            float prefix = 0.0f;
            for (int b2 = 0; b2 < b; ++b2) prefix = __fadd_rn(prefix, sh.sbs[b2]);
            if (__fadd_rn(prefix, sh.sbs[b]) > target) {
              float run = prefix;
              for (int i = b * ACC_BLK; i < V && i < (b + 1) * ACC_BLK; ++i) {
                run = __fadd_rn(run, sh.blk[kb][i - b * ACC_BLK]);
                if (run > target) { atomicMin(&G->pick, (unsigned)i); break; }
              }
            }
          }
        }
        if (!(ok = acc_grid_sync(G, ++gen, A.err, sh))) break;
        const unsigned pk = __ldcg(&G->pick);
        int pick = (int)pk;
        if (pk == 0xFFFFFFFFu) {
          int hi = -1;
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
            if (idk[kb] < V && pv[kb] > 0.0f) hi = max(hi, idk[kb]);
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, off));
          if (lane == 0 && hi >= 0) atomicMax(&G->hi, hi);
          if (!(ok = acc_grid_sync(G, ++gen, A.err, sh))) break;
          const int h = __ldcg(&G->hi);
          pick = h < 0 ? 0 : h;
        }
        if (writer) A.out[no] = pick;
        ++no;
        break;
      }
    }
    if (writer) {
      A.out[no] = A.tokens[acc];
      A.path[np] = acc;
    }
    ++no;
    ++np;
    v = acc;
  }
  if (writer) {
    A.count[0] = ok ? no : 0;
    A.count[1] = ok ? np : 0;
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
