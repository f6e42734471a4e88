// kq_batch.cuh -- a forward pass over M <= 64 tokens at once (the verification pass over a draft
// tree), so the weights stream from HBM once per pass instead of once per node.
//
//  * k_mm: fused-dequant GEMM Y[M][R] = X[M][C] W^T on the tensor cores (mma.sync m16n8k16,
//    fp32 accumulation) with split-precision fp16 operands: every weight w (dequantised in fp32:
//    w = d*sc*q - dmin*mn, or d*scale*(q6 - 32)) and every activation x are carried as
//    hi = fp16(v) plus lo = fp16(v - hi), and each tile takes three products (hi*hi, hi*lo,
//    lo*hi), about 22 significant bits, so the result is within fp32 rounding of an fp32 GEMM. A
//    warp owns 16 weight rows (two 8-row tiles of the kq layout) for all M tokens; it reads its
//    rows' bytes straight from global memory and dequantises them in registers into the A
//    fragments; the CTA stages X one 256-column super-block at a time in shared memory (hi and lo
//    planes) for the B fragments. Epilogues per (row, token): fp32 store, NeoX rotary (q to fp32,
//    k to the fp16 cache at the token's slot), V store, SwiGLU. This is the small-M path
//    (M = 2..64); the M = 1 decode keeps the exact digit-plane GEMV of kq_gemv.cuh.
//  * k_bnorm: per token, the residual add and fp64-sum RMS norm (or the embedding row), writing
//    h and the (fp32) input of the next GEMM.
//  * k_battn: attention of all tokens of the pass over the cache prefix and the tree slots, with
//    each token's ancestor mask; CTA (kv head, position split, block of 16 tokens), the partials
//    merged in split order by the last CTA of each (kv head, token block).
#pragma once
#include "kq_common.cuh"
#include "kq_qformat.cuh"
#include "kq_gemv.cuh"
#include <cfloat>

namespace kq {

constexpr int MM_MAXM = 64;            // tokens per pass (8 n-tiles of 8)
constexpr int MM_WARPS = 4;            // warps per CTA, 16 rows each
constexpr int MM_XPAD = 8;             // fp16 padding of a staged X row (conflict-free B loads)

struct BatchParams {                   // per-token data of a pass
  int M;
  const int* slot;                     // [M] K/V slot
  const int* rpos;                     // [M] rotary position
  const unsigned long long* mask;      // [M][2] ancestor masks relative to tree_base
  int tree_base;
};

struct MMParams {
  Seg seg[KQ_MAX_SEG];                 // rows of segment i: seg[i].w.R (multiples of 16)
  int nseg;
  int C, G;
  const float* X;                      // [M][C]
  BatchParams B;
  int out_ld;                          // row length of fp32 / fp16 outputs (per segment: see epi)
  const float* cos_t;
  const float* sin_t;
  int hd, ctx;
};

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  hi = h2u(h);
  lo = h2u(__floats2half2_rn(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y)));
}

// The two weights of a row at K-step columns (j, j + 1) of a 16-column half sub-block, from the
// 16 nibble / ql bytes of that half (bytes j, j + 1 of `w4`), as hi / lo fp16 pairs. Q4_K: value
// nibble `hi`, w = d*sc*q - dmin*mn (the reference order, q4kernels.h:19-21).
__device__ __forceinline__ void dq_q4k_pair(const uint32_t (&w4)[4], int j, int nib, float ds, float dm, uint32_t& hi,
                                            uint32_t& lo) {
  const uint32_t word = w4[j >> 2];
  const int sh = (j & 3) * 8 + nib * 4;
  const float q0 = (float)((word >> sh) & 15u), q1 = (float)((word >> (sh + 8)) & 15u);
  split_h2(__fsub_rn(__fmul_rn(ds, q0), dm), __fsub_rn(__fmul_rn(ds, q1), dm), hi, lo);
}
// Q6_K: w = (d*scale) * (q6 - 32) (q4kernels.h:29-30)
__device__ __forceinline__ void dq_q6k_pair(const uint32_t (&l4)[4], const uint32_t (&h4)[4], int j, int k, float dsc,
                                            uint32_t& hi, uint32_t& lo) {
  const uint32_t lw = l4[j >> 2], hw = h4[j >> 2];
  const int sh = (j & 3) * 8;
  const int lsh = (k >> 1) * 4, hsh = 2 * k;
  const int q0 = (int)(((lw >> sh) >> lsh) & 15u) | (int)((((hw >> sh) >> hsh) & 3u) << 4);
  const int q1 = (int)(((lw >> (sh + 8)) >> lsh) & 15u) | (int)((((hw >> (sh + 8)) >> hsh) & 3u) << 4);
  split_h2(__fmul_rn(dsc, (float)(q0 - 32)), __fmul_rn(dsc, (float)(q1 - 32)), hi, lo);
}

__device__ __forceinline__ uint4 ldg16(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

constexpr size_t MM_SMEM = (size_t)2 * MM_MAXM * (256 + MM_XPAD) * 2;   // hi and lo planes of X

__global__ void __launch_bounds__(MM_WARPS * 32) k_mm(const __grid_constant__ MMParams P) {
  extern __shared__ __align__(16) uint8_t mm_smem[];
  __half (*xs)[256 + MM_XPAD] = reinterpret_cast<__half (*)[256 + MM_XPAD]>(mm_smem);                 // hi
  __half (*xl)[256 + MM_XPAD] = reinterpret_cast<__half (*)[256 + MM_XPAD]>(mm_smem + MM_SMEM / 2);   // lo
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, grp = lane >> 2, t4 = lane & 3;
  const int M = P.B.M, ntiles = (M + 7) >> 3, G = P.G;
  // this warp's 16 rows: segment and local row
  int row0 = (blockIdx.x * MM_WARPS + warp) * 16, segi = 0;
  while (segi < P.nseg && row0 >= P.seg[segi].w.R) { row0 -= P.seg[segi].w.R; ++segi; }
  const bool active = segi < P.nseg;
  const Seg& sg = P.seg[active ? segi : 0];
  const QView& w = sg.w;
  const bool q4 = w.type == Q4K;
  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  for (int g = 0; g < G; ++g) {
    __syncthreads();
    // X[:, 256g .. 256g + 255] -> hi / lo planes (tokens past M as zeros)
    for (int i = threadIdx.x; i < ntiles * 8 * 64; i += MM_WARPS * 32) {
      const int tk = i >> 6, c4 = i & 63;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (tk < M) v = __ldg(reinterpret_cast<const float4*>(P.X + (size_t)tk * P.C + 256 * g + 4 * c4));
      uint32_t h0, l0, h1, l1;
      split_h2(v.x, v.y, h0, l0);
      split_h2(v.z, v.w, h1, l1);
      *reinterpret_cast<uint2*>(&xs[tk][4 * c4]) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(&xl[tk][4 * c4]) = make_uint2(l0, l1);
    }
    __syncthreads();
    if (!active) continue;
    // per row (grp, grp + 8): block header of super-block g
    const int rA = row0 + grp, rB = row0 + 8 + grp;
    float dsA[8], dmA[8], dsB[8], dmB[8];   // Q4_K: d*sc, dmin*mn per sub-block ; Q6_K: d in ds[0]
    if (q4) {
      const uint4 MA = ldg16(w.base + row_plane_off(Q4K, G, rA, 1, (size_t)g * 16));
      const uint4 MB = ldg16(w.base + row_plane_off(Q4K, G, rB, 1, (size_t)g * 16));
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t scA, mnA, scB, mnB;
        q4k_scale_words(MA, hh, scA, mnA);
        q4k_scale_words(MB, hh, scB, mnB);
        const float dA = h2f_bits(MA.x & 0xFFFFu), dminA = h2f_bits(MA.x >> 16);
        const float dB = h2f_bits(MB.x & 0xFFFFu), dminB = h2f_bits(MB.x >> 16);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          dsA[4 * hh + k] = __fmul_rn(dA, (float)((scA >> (8 * k)) & 0xFF));
          dmA[4 * hh + k] = __fmul_rn(dminA, (float)((mnA >> (8 * k)) & 0xFF));
          dsB[4 * hh + k] = __fmul_rn(dB, (float)((scB >> (8 * k)) & 0xFF));
          dmB[4 * hh + k] = __fmul_rn(dminB, (float)((mnB >> (8 * k)) & 0xFF));
        }
      }
    } else {
      const size_t dA = row_plane_off(Q6K, G, rA, 3, (size_t)g * 2), dB = row_plane_off(Q6K, G, rB, 3, (size_t)g * 2);
      dsA[0] = __half2float(*reinterpret_cast<const __half*>(w.base + dA));
      dsB[0] = __half2float(*reinterpret_cast<const __half*>(w.base + dB));
    }
    // the 16 K-steps of the super-block: unit u = 2h + jh, sub-block k (Q4_K: chunk c = (k/2)%2,
    // nibble k%2 of sub-block 4h + k ; Q6_K: ql chunk k%2, nibble k/2, qh shift 2k)
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int hh = u >> 1, jh = u & 1;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t wA[4], wB[4];
        {
          const uint4 A = ldg16(w.base + row_plane_off(w.type, G, rA, 0, (size_t)c * 64 * G + (size_t)g * 64 + u * 16));
          const uint4 Bv = ldg16(w.base + row_plane_off(w.type, G, rB, 0, (size_t)c * 64 * G + (size_t)g * 64 + u * 16));
          wA[0] = A.x; wA[1] = A.y; wA[2] = A.z; wA[3] = A.w;
          wB[0] = Bv.x; wB[1] = Bv.y; wB[2] = Bv.z; wB[3] = Bv.w;
        }
        uint32_t hA[4] = {0, 0, 0, 0}, hB[4] = {0, 0, 0, 0};
        uint32_t scA = 0, scB = 0;
        if (!q4) {
          const uint4 A = ldg16(w.base + row_plane_off(Q6K, G, rA, 1, (size_t)g * 64 + u * 16));
          const uint4 Bv = ldg16(w.base + row_plane_off(Q6K, G, rB, 1, (size_t)g * 64 + u * 16));
          hA[0] = A.x; hA[1] = A.y; hA[2] = A.z; hA[3] = A.w;
          hB[0] = Bv.x; hB[1] = Bv.y; hB[2] = Bv.z; hB[3] = Bv.w;
          scA = __ldg(reinterpret_cast<const uint32_t*>(w.base + row_plane_off(Q6K, G, rA, 2, (size_t)g * 16 + u * 4)));
          scB = __ldg(reinterpret_cast<const uint32_t*>(w.base + row_plane_off(Q6K, G, rB, 2, (size_t)g * 16 + u * 4)));
        }
#pragma unroll
        for (int nib = 0; nib < 2; ++nib) {
          // Q4_K: sub-block 4h + 2c + nib ; Q6_K: k = c + 2 * nib
          const int kq4 = 2 * c + nib, k6 = c + 2 * nib;
          const int col0 = q4 ? 128 * hh + 32 * kq4 + 16 * jh : 128 * hh + 32 * k6 + 16 * jh;
          uint32_t a[4], al[4];
          if (q4) {
            const float sA = dsA[4 * hh + kq4], mA = dmA[4 * hh + kq4], sB = dsB[4 * hh + kq4], mB = dmB[4 * hh + kq4];
            dq_q4k_pair(wA, 2 * t4, nib, sA, mA, a[0], al[0]);
            dq_q4k_pair(wB, 2 * t4, nib, sB, mB, a[1], al[1]);
            dq_q4k_pair(wA, 2 * t4 + 8, nib, sA, mA, a[2], al[2]);
            dq_q4k_pair(wB, 2 * t4 + 8, nib, sB, mB, a[3], al[3]);
          } else {
            const float sA = __fmul_rn(dsA[0], (float)(int8_t)((scA >> (8 * k6)) & 0xFF));
            const float sB = __fmul_rn(dsB[0], (float)(int8_t)((scB >> (8 * k6)) & 0xFF));
            dq_q6k_pair(wA, hA, 2 * t4, k6, sA, a[0], al[0]);
            dq_q6k_pair(wB, hB, 2 * t4, k6, sB, a[1], al[1]);
            dq_q6k_pair(wA, hA, 2 * t4 + 8, k6, sA, a[2], al[2]);
            dq_q6k_pair(wB, hB, 2 * t4 + 8, k6, sB, a[3], al[3]);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (j < ntiles) {
              const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&xs[8 * j + grp][col0 + 2 * t4]);
              const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&xs[8 * j + grp][col0 + 2 * t4 + 8]);
              const uint32_t c0 = *reinterpret_cast<const uint32_t*>(&xl[8 * j + grp][col0 + 2 * t4]);
              const uint32_t c1 = *reinterpret_cast<const uint32_t*>(&xl[8 * j + grp][col0 + 2 * t4 + 8]);
              mma16816(acc[j], al, b0, b1);   // small terms first
              mma16816(acc[j], a, c0, c1);
              mma16816(acc[j], a, b0, b1);
            }
          }
        }
      }
    }
  }
  if (!active) return;
  // ---- epilogue: acc[j] = D[row grp / grp + 8][tokens 8j + 2t4, + 1]
  const int epi = sg.epi;
  const bool pair = epi == EPI_ROPE_Q || epi == EPI_ROPE_K || epi == EPI_SWIGLU;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j >= ntiles) break;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float v = acc[j][e];
      const float vo = pair ? __shfl_xor_sync(0xffffffffu, v, 4) : 0.f;   // row r ^ 1
      const int r = row0 + grp + ((e >> 1) << 3);
      const int tk = 8 * j + 2 * t4 + (e & 1);
      if (tk >= M) continue;
      switch (epi) {
        case EPI_F32:
          sg.out_f[(size_t)tk * P.out_ld + r] = v;
          break;
        case EPI_V: {
          const int kv = r / P.hd, d = r % P.hd;
          sg.out_h[((size_t)kv * P.ctx + P.B.slot[tk]) * P.hd + d] = __float2half_rn(v);
        } break;
        case EPI_SWIGLU:   // the down GEMM's input, [M][out_ld]
          if ((grp & 1) == 0) sg.out_f[(size_t)tk * P.out_ld + (r >> 1)] = __fmul_rn(silu_f(v), vo);
          break;
        case EPI_ROPE_Q:
        case EPI_ROPE_K:
          if ((grp & 1) == 0) {
            const int hh = r / P.hd, i2 = (r % P.hd) >> 1, half = P.hd >> 1;
            const int rp = P.B.rpos[tk];
            const float cs = __ldg(P.cos_t + (size_t)rp * half + i2), sn = __ldg(P.sin_t + (size_t)rp * half + i2);
            const float o0 = __fsub_rn(__fmul_rn(v, cs), __fmul_rn(vo, sn));
            const float o1 = __fadd_rn(__fmul_rn(v, sn), __fmul_rn(vo, cs));
            if (epi == EPI_ROPE_Q) {
              float* q = sg.out_f + (size_t)tk * P.out_ld + (size_t)hh * P.hd;
              q[i2] = o0;
              q[i2 + half] = o1;
            } else {
              __half* dst = sg.out_h + ((size_t)hh * P.ctx + P.B.slot[tk]) * P.hd;
              dst[i2] = __float2half_rn(o0);
              dst[i2 + half] = __float2half_rn(o1);
            }
          }
          break;
      }
    }
  }
}

// ------------------------------------------------------------------------------ norm / embedding
struct BNormParams {
  int M, D;
  const int* tok;          // [M] (embedding mode)
  QView emb;               // embedding matrix, or type 0: residual mode
  float* h;                // [M][D] residual stream (read-modify-write)
  const float* y;          // [M][D] block output to add (residual mode), or null
  const float* gamma;      // [D]
  float eps;
  float* X;                // [M][D] normed input of the next GEMM
  int vocab;
  int* err;
};
__global__ void __launch_bounds__(256) k_bnorm(const __grid_constant__ BNormParams P) {
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ double red[8];
  float* h = P.h + (size_t)t * P.D;
  double acc = 0.0;
  if (P.emb.base) {
    int tok = P.tok[t];
    if (tok < 0 || tok >= P.vocab) {
      if (tid == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_TOKEN);
      tok = 0;
    }
    for (int i = tid; i < P.D; i += 256) {
      const float v = dequant_elem(P.emb, tok, i);
      h[i] = v;
      acc = __dadd_rn(acc, __dmul_rn((double)v, (double)v));
    }
  } else {
    for (int i = tid; i < P.D; i += 256) {
      const float v = P.y ? __fadd_rn(h[i], P.y[(size_t)t * P.D + i]) : h[i];
      h[i] = v;
      acc = __dadd_rn(acc, __dmul_rn((double)v, (double)v));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  double tot = 0.0;
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / (double)P.D), P.eps)));
  for (int i = tid; i < P.D; i += 256)
    P.X[(size_t)t * P.D + i] = __fmul_rn(__fmul_rn(h[i], s), P.gamma[i]);
}

// ------------------------------------------------------------------------------ tree attention
constexpr int BA_TOK = 16;           // tokens per CTA
constexpr int BA_CH = 32;            // positions per chunk
constexpr int BA_THREADS = 256;

struct BAttnParams {
  const float* q;                    // [M][NH * HD] rotated queries
  const __half* kc;                  // [n_kv][ctx][HD]
  const __half* vc;
  float* out;                        // [M][NH * HD] (the o GEMM's input)
  BatchParams B;
  int n_kv, G, ctx, npos;            // npos: slots [0, npos) may be attended
  float scale;
  int nsplit;
  float* part;                       // [n_kv][tokblocks][nsplit][BA_TOK * G][HD + 2]
  int* ticket;                       // [n_kv][tokblocks]
};

// CTA (kv head, split, token block): the block's BA_TOK tokens x G heads against the positions
// of the split, chunk by chunk; online softmax per query; partial (m, l, o) to scratch; the last
// CTA of (kv head, token block) merges the splits in order and writes fp16 outputs.
template <int G>
__global__ void __launch_bounds__(BA_THREADS) k_battn(const __grid_constant__ BAttnParams P) {
  constexpr int HD = 128, NQ = BA_TOK * G;
  extern __shared__ __align__(16) uint8_t sm[];
  float* qs = reinterpret_cast<float*>(sm);                       // [NQ][HD]
  float* os = qs + NQ * HD;                                       // [NQ][HD] accumulators
  float* ss = os + NQ * HD;                                       // [NQ][BA_CH] scores
  float* mrow = ss + NQ * BA_CH;                                  // [NQ] running max
  float* lrow = mrow + NQ;                                        // [NQ] running sum
  float* frow = lrow + NQ;                                        // [NQ] rescale of this chunk
  __half* ks = reinterpret_cast<__half*>(frow + NQ);              // [BA_CH][HD]
  __half* vs = ks + BA_CH * HD;                                   // [BA_CH][HD]
  __shared__ int s_last;
  const int kv = blockIdx.x, sp = blockIdx.y, tb = blockIdx.z, tid = threadIdx.x;
  const int M = P.B.M, tok0 = tb * BA_TOK, ntok = min(BA_TOK, M - tok0);
  const int tokblocks = (M + BA_TOK - 1) / BA_TOK;
  const int per = (P.npos + P.nsplit - 1) / P.nsplit;
  const int p0 = min(P.npos, sp * per), p1 = min(P.npos, p0 + per);
  const int NHHD = P.n_kv * G * HD;
  for (int i = tid; i < NQ * HD; i += BA_THREADS) {
    const int qi = i / HD, d = i % HD, tk = qi / G, gh = qi % G;
    qs[i] = tk < ntok ? P.q[(size_t)(tok0 + tk) * NHHD + (size_t)(kv * G + gh) * HD + d] : 0.f;
    os[i] = 0.f;
  }
  for (int i = tid; i < NQ; i += BA_THREADS) { mrow[i] = -FLT_MAX; lrow[i] = 0.f; }
  __syncthreads();
  const __half* kb = P.kc + (size_t)kv * P.ctx * HD;
  const __half* vb = P.vc + (size_t)kv * P.ctx * HD;
  for (int c0 = p0; c0 < p1; c0 += BA_CH) {
    const int cnt = min(BA_CH, p1 - c0);
    for (int i = tid; i < cnt * HD / 8; i += BA_THREADS) {
      reinterpret_cast<uint4*>(ks)[i] = __ldcg(reinterpret_cast<const uint4*>(kb + (size_t)c0 * HD) + i);
      reinterpret_cast<uint4*>(vs)[i] = __ldcg(reinterpret_cast<const uint4*>(vb + (size_t)c0 * HD) + i);
    }
    __syncthreads();
    // scores: thread -> (query, position) pairs
    for (int e = tid; e < NQ * BA_CH; e += BA_THREADS) {
      const int qi = e / BA_CH, pp = e % BA_CH, tk = qi / G;
      float a = -INFINITY;
      if (pp < cnt && tk < ntok) {
        const int t = c0 + pp, gt = tok0 + tk;
        const bool vis = t < P.B.tree_base ||
                         slot_attended(t, P.B.tree_base, P.B.mask[2 * gt], P.B.mask[2 * gt + 1]);
        if (vis) {
          const float* q = qs + qi * HD;
          const __half2* k2 = reinterpret_cast<const __half2*>(ks + pp * HD);
          float s = 0.f;
#pragma unroll 8
          for (int d2 = 0; d2 < HD / 2; ++d2) {
            const float2 kf = __half22float2(k2[d2]);
            s = __fmaf_rn(kf.x, q[2 * d2], s);
            s = __fmaf_rn(kf.y, q[2 * d2 + 1], s);
          }
          a = __fmul_rn(s, P.scale);
        }
      }
      ss[e] = a;
    }
    __syncthreads();
    // online softmax per query (one warp per query, round-robin)
    for (int qi = tid >> 5; qi < NQ; qi += BA_THREADS / 32) {
      const int lane = tid & 31;
      float m = -FLT_MAX;
      for (int pp = lane; pp < BA_CH; pp += 32) m = fmaxf(m, ss[qi * BA_CH + pp]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      const float m_old = mrow[qi], m_new = fmaxf(m_old, m);
      float l = 0.f;
      for (int pp = lane; pp < BA_CH; pp += 32) {
        const float ev = expf(__fsub_rn(ss[qi * BA_CH + pp], m_new));
        ss[qi * BA_CH + pp] = ev;
        l += ev;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) {
        const float f = expf(__fsub_rn(m_old, m_new));
        frow[qi] = f;
        lrow[qi] = __fmaf_rn(lrow[qi], f, l);
        mrow[qi] = m_new;
      }
    }
    __syncthreads();
    // P.V: thread -> (query, dim) accumulators
    for (int e = tid; e < NQ * HD; e += BA_THREADS) {
      const int qi = e / HD, d = e % HD;
      float o = __fmul_rn(os[e], frow[qi]);
      for (int pp = 0; pp < cnt; ++pp) o = __fmaf_rn(ss[qi * BA_CH + pp], __half2float(vs[pp * HD + d]), o);
      os[e] = o;
    }
    __syncthreads();
  }
  // ---- partial to scratch: [kv][tb][sp][qi][HD + 2]
  const size_t base = (((size_t)kv * tokblocks + tb) * P.nsplit + sp) * NQ * (HD + 2);
  for (int e = tid; e < NQ * HD; e += BA_THREADS) {
    const int qi = e / HD, d = e % HD;
    __stcg(P.part + base + (size_t)qi * (HD + 2) + d, os[e]);
  }
  for (int qi = tid; qi < NQ; qi += BA_THREADS) {
    __stcg(P.part + base + (size_t)qi * (HD + 2) + HD, mrow[qi]);
    __stcg(P.part + base + (size_t)qi * (HD + 2) + HD + 1, lrow[qi]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&P.ticket[kv * tokblocks + tb], 1) == P.nsplit - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- merge the splits in order
  const size_t b0 = ((size_t)kv * tokblocks + tb) * P.nsplit * NQ * (HD + 2);
  for (int e = tid; e < NQ * HD; e += BA_THREADS) {
    const int qi = e / HD, d = e % HD, tk = qi / G, gh = qi % G;
    if (tk >= ntok) continue;
    float Mx = -FLT_MAX;
    for (int s2 = 0; s2 < P.nsplit; ++s2) Mx = fmaxf(Mx, __ldcg(P.part + b0 + ((size_t)s2 * NQ + qi) * (HD + 2) + HD));
    float L = 0.f, O = 0.f;
    for (int s2 = 0; s2 < P.nsplit; ++s2) {
      const float* pr = P.part + b0 + ((size_t)s2 * NQ + qi) * (HD + 2);
      const float wgt = expf(__fsub_rn(__ldcg(pr + HD), Mx));
      L = __fmaf_rn(wgt, __ldcg(pr + HD + 1), L);
      O = __fmaf_rn(wgt, __ldcg(pr + d), O);
    }
    P.out[(size_t)(tok0 + tk) * NHHD + (size_t)(kv * G + gh) * HD + d] = __fdiv_rn(O, L);
  }
  if (tid == 0) P.ticket[kv * tokblocks + tb] = 0;
}

__host__ __device__ inline size_t battn_smem(int G) {
  const int NQ = BA_TOK * G;
  return (size_t)(2 * NQ * 128 + NQ * BA_CH + 3 * NQ) * 4 + (size_t)2 * BA_CH * 128 * 2;
}

// Per-token argmax of the logits (lowest index on ties), one CTA per token.
__global__ void __launch_bounds__(256) k_argmax_rows(const float* logits, int V, int* out) {
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float bv[8];
  __shared__ int bi[8];
  float v = -INFINITY;
  int vi = 0x7fffffff;
  const float* z = logits + (size_t)t * V;
  for (int i = tid; i < V; i += 256) {
    const float x = z[i];
    if (x > v || (x == v && i < vi)) { v = x; vi = i; }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, off);
    const int oi = __shfl_xor_sync(0xffffffffu, vi, off);
    if (ov > v || (ov == v && oi < vi)) { v = ov; vi = oi; }
  }
  if (lane == 0) { bv[warp] = v; bi[warp] = vi; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < 8; ++w)
      if (bv[w] > v || (bv[w] == v && bi[w] < vi)) { v = bv[w]; vi = bi[w]; }
    out[t] = vi == 0x7fffffff ? 0 : vi;
  }
}

}  // namespace kq
