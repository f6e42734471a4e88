// kq_gemv.cuh -- fused-dequant Q4_K / Q6_K GEMV for single-token decode on sm_100a.
//
// Replaces the reference's q4_gemv (scripts/kindi_q4/kindi/q4.cu:18-27), q4_embed (:28-32),
// q4_rms (:39-46) and q4_silu (:36-38), and the rope / K-V store of engine.py:260-267.
//
// Design:
//  * Persistent CTAs (one per SM). A producer warp streams "stages" of TR rows (whole 8-row tiles
//    of the kq layout, so ONE contiguous 1-D bulk copy per stage, cp.async.bulk with L2
//    evict-first) into a shared-memory ring; completion is tracked by mbarriers. The producer
//    starts before griddepcontrol.wait, so the weight stream of kernel N+1 starts while kernel N
//    finishes.
//  * Activations: in the prologue the CTA splits its fp32 activation vector exactly into three
//    int8 digit planes, x = s1*x1 + s2*x2 + s3*x3 per 64-column "unit" (s1 a power of two with
//    max|x| <= 127*s1, s2 = s1/128, s3 = s1/16384; residual <= s1/32768), stored in shared
//    memory as [group k][plane][unit] (conflict-free 16-byte reads).
//  * Consumers: thread u of a row group owns unit u (64 columns, see kq_qformat.cuh) and RPG rows
//    of every stage. Dot products of the 4-/6-bit weights with the digit planes are exact int32
//    dp4a sums per 16-element group, multiplied by the integer block scales in int32; the three
//    planes are combined once per row in fp32. Row partials are reduced with a fixed warp-shuffle
//    tree, then across the row's warps in a fixed order (one named barrier per stage), so results
//    do not depend on timing.
//  * Fusions: prologue = residual add + fp64 RMS norm (q4_rms) or embedding-row dequantisation
//    (q4_embed); epilogue = NeoX rotary + fp16 K/V store, V store, SwiGLU, or the output-head
//    argmax with a last-CTA merge (lowest index on ties, like k_argmax kindi.cu:637-661).
#pragma once
#include "kq_common.cuh"
#include "kq_qformat.cuh"
#include <cfloat>

namespace kq {

enum { EPI_F32 = 0, EPI_ROPE_Q = 1, EPI_ROPE_K = 2, EPI_V = 3, EPI_SWIGLU = 4, EPI_ARGMAX = 5 };
enum { XS_PLAIN = 0, XS_NORM = 1, XS_EMBED = 2 };
enum { TM_Q4K = 1, TM_Q6K = 2, TM_MIXED = 3 };
constexpr int KQ_MAX_SEG = 4;
constexpr int KQ_GEMV_MAX_CONSUMERS = 384;
constexpr int KQ_GEMV_MAX_THREADS = KQ_GEMV_MAX_CONSUMERS + 32;   // + one producer warp
constexpr int KQ_MAX_NRG = 8;              // row groups (named barriers 1..8)
constexpr int KQ_BAR_PROLOGUE = 14, KQ_BAR_ARGMAX = 15;
constexpr int KQ_XSCAL = 18;               // per-unit scalars: s3, poison, xsf[4], c[3][4]
constexpr int KQ_MAX_ITEMS = 4;            // prologue items per thread: the planner keeps >= 2 row groups
constexpr int KQ_MAX_HALF_HD = 128;        // rotary half width held in shared memory
// Stages the producer issues before the consumers' prologue is done (the ring holds >= 2).
// Measured on the config-0 GEMV / config-2 decode step: 1 stage 12.1 us / 2.62 ms, 2 stages
// 12.05 us / 2.57 ms, the whole ring (3 slots) 13.0 us / 2.58 ms.
constexpr int KQ_PREFETCH_STAGES = 2;
constexpr int KQ_MAX_SLOTS = 8;             // ring slots of a GEMV kernel at most (the planners' cap)

struct DecodeState {   // device-resident per-step state
  int tok;        // token processed by this step
  int pos;        // its K/V slot (its position, for a plain decode step)
  int next_tok;   // argmax written by the output head
  int steps;      // steps completed by the device-resident loop
  int rpos;       // position of its rotary angle (pos, except for draft-tree nodes)
  int tree_base;  // slots below tree_base are all attended; slot tree_base + j only if bit j of
  int pad;        // mask is set (a draft tree's ancestors and the node itself); pos + 1 when
  unsigned long long mask[2];   // there is no tree
};

// Attention visibility of cache slot t for the step described by (tree_base, mask).
__device__ __forceinline__ bool slot_attended(int t, int tree_base, unsigned long long m0, unsigned long long m1) {
  if (t < tree_base) return true;
  const int j = t - tree_base;
  return j < 128 && (((j < 64 ? m0 : m1) >> (j & 63)) & 1ull);
}

struct Seg {
  QView w;
  int stage0, nstage;   // global stage range of this segment
  int tr;               // rows per stage (whole 8-row tiles; the last stage may be shorter)
  int epi;
  float* out_f;         // F32 / ROPE_Q / SWIGLU / ARGMAX (logits)
  __half* out_h;        // ROPE_K / V: this layer's cache [n_kv][ctx][hd]
};

struct GemvParams {
  Seg seg[KQ_MAX_SEG];
  int nseg, nstages;
  int C, G, TR, LPR, NRG;
  int nlanes;            // independent thread lanes (the persistent kernel; 1 for k_gemv), each
                         // LPR * NRG threads consuming its own stages
  int tps;               // persistent kernel: stages (of TR rows) per ring entry
  int stage_bytes, nslots;
  // activation source
  int xmode;
  const float* x;
  const float* h_in;
  const float* y_add;
  const float* gamma;
  float* h_out;
  float eps;
  QView emb;
  DecodeState* st;
  int vocab;
  // epilogue auxiliaries
  const float* cos_t;
  const float* sin_t;
  int hd, ctx;
  float* part_val;
  int* part_idx;
  int* ticket;
  int* out_ids;          // ARGMAX: token of step st->steps is written here (device loop)
  int out_cap;
  int* err;
  int trace_id;          // launch index for the optional phase trace (KQ_TRACE builds)
  int prefetch;          // k_gemv: stages the producer issues before the consumers' prologue is done
  int* dyn;              // {next stage, CTAs done claiming}, zero between launches: every CTA's
                         // producer claims its stages at run time, one ahead (null: fixed ranges)
};

// Shared-memory carve-up, identical on host (sizing) and device.
struct GemvSmem {
  size_t stages, xplanes, xscal, bars, red, redd, best, rope, total;
};
__host__ __device__ inline size_t gs_align(size_t x, size_t a) { return (x + a - 1) / a * a; }
__host__ __device__ inline GemvSmem gemv_smem_layout(int nslots, int stage_bytes, int LPR, int NRG, int RPG, int nthr_c) {
  GemvSmem s;
  const int WPR = LPR >= 32 ? LPR / 32 : 1;
  size_t o = 0;
  s.stages = o; o += (size_t)nslots * stage_bytes;
  s.xplanes = o = gs_align(o, 128); o += (size_t)12 * LPR * 16;
  s.xscal = o = gs_align(o, 16); o += (size_t)KQ_XSCAL * LPR * 4;
  s.bars = o = gs_align(o, 8); o += (size_t)2 * nslots * 8;
  s.red = o = gs_align(o, 8); o += (size_t)2 * RPG * NRG * WPR * 4;
  s.redd = o = gs_align(o, 8); o += (size_t)((nthr_c + 31) / 32) * 8;
  s.best = o = gs_align(o, 8); o += (size_t)NRG * RPG * 8;
  s.rope = o = gs_align(o, 16); o += (size_t)2 * KQ_MAX_HALF_HD * 4;   // cos, sin of this step's position
  s.total = gs_align(o, 128);
  return s;
}

__device__ __forceinline__ float pow2f(int k) { return __int_as_float((k + 127) << 23); }

__device__ __forceinline__ float byte_to_float_u(uint32_t w, int i) {
  return __fsub_rn(__int_as_float((int)__byte_perm(w, 0x4B000000u, (uint32_t)(i | 0x7440))), 8388608.f);
}

// Per-unit activation scalars held in registers by a consumer thread.
struct XS {
  float s3, poison;
  float xsf[4];     // sum of group k's digits 16384*S1 + 128*S2 + S3, as float (Q4_K dmin term)
  int c[3][4];      // 32 * (sum of plane L's digits of group k): the "-32" of Q6_K, exact
};

// ------------------------------------------------------------------------------ row math
// dp4a with unsigned bytes in a (weights) and signed bytes in b (activation digits).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int sbyte(uint32_t w, int k) {   // sign-extended byte k
  return ((int)(w << (24 - 8 * k))) >> 24;
}

// Q4_K, group k of a unit, all three digit planes: P[L] += c_k * sum_j q_j * xL_j with
// c_k = 16 sc_k for the low-nibble groups (k even) and sc_k for the high-nibble groups, whose
// bytes are used in place (16 q_j = w & 0xF0F0F0F0). So P[L] = 16 * sum_k sc_k * sum_j q_j xL_j,
// exact in int32 (|P| < 1.3e8).
__device__ __forceinline__ void q4k_group(const uint32_t (&src)[4], int k, uint32_t sc_w, const uint4 (&xw)[3], int (&P)[3]) {
  const uint32_t msk = (k & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
  const uint32_t x0[4] = {xw[0].x, xw[0].y, xw[0].z, xw[0].w};
  const uint32_t x1[4] = {xw[1].x, xw[1].y, xw[1].z, xw[1].w};
  const uint32_t x2[4] = {xw[2].x, xw[2].y, xw[2].z, xw[2].w};
  int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t nib = src[i] & msk;
    s0 = dp4a_us(nib, x0[i], s0);
    s1 = dp4a_us(nib, x1[i], s1);
    s2 = dp4a_us(nib, x2[i], s2);
  }
  const int ck = (int)((sc_w >> (8 * k)) & 0xFFu) << ((k & 1) ? 0 : 4);
  P[0] += ck * s0;
  P[1] += ck * s1;
  P[2] += ck * s2;
}
// Q6_K, group k: P[L] += scale_k * (sum_j q6_j * xL_j - 32 * sum_j xL_j), exact in int32.
__device__ __forceinline__ void q6k_group(const uint32_t (&a)[4], const uint32_t (&b)[4], const uint32_t (&q)[4], int k,
                                          uint32_t scw, const uint4 (&xw)[3], const XS& xs, int (&P)[3]) {
  const uint32_t x0[4] = {xw[0].x, xw[0].y, xw[0].z, xw[0].w};
  const uint32_t x1[4] = {xw[1].x, xw[1].y, xw[1].z, xw[1].w};
  const uint32_t x2[4] = {xw[2].x, xw[2].y, xw[2].z, xw[2].w};
  int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t srcw = (k & 1) ? b[i] : a[i];
    const uint32_t lo = (k >> 1) ? ((srcw >> 4) & 0x0F0F0F0Fu) : (srcw & 0x0F0F0F0Fu);
    const uint32_t hi = (k == 0) ? ((q[i] << 4) & 0x30303030u)
                      : (k == 1) ? ((q[i] << 2) & 0x30303030u)
                      : (k == 2) ? (q[i] & 0x30303030u)
                                 : ((q[i] >> 2) & 0x30303030u);
    const uint32_t q6 = lo | hi;
    s0 = dp4a_us(q6, x0[i], s0);
    s1 = dp4a_us(q6, x1[i], s1);
    s2 = dp4a_us(q6, x2[i], s2);
  }
  const int sk = sbyte(scw, k);
  P[0] += sk * (s0 - xs.c[0][k]);
  P[1] += sk * (s1 - xs.c[1][k]);
  P[2] += sk * (s2 - xs.c[2][k]);
}
// The three planes' integer sums combined in fp32: 16384 P0 + 128 P1 + P2 (two roundings).
__device__ __forceinline__ float planes_combine(const int (&P)[3]) {
  return __fmaf_rn((float)P[0], 16384.f, __fmaf_rn((float)P[1], 128.f, (float)P[2]));
}

// Six-bit scales / mins of sub-blocks 4h .. 4h+3 as four bytes each (q4kernels.h:17-18).
__device__ __forceinline__ void q4k_scale_words(const uint4 meta, int h, uint32_t& sc_w, uint32_t& mn_w) {
  sc_w = h ? ((meta.w & 0x0F0F0F0Fu) | ((meta.y >> 2) & 0x30303030u)) : (meta.y & 0x3F3F3F3Fu);
  mn_w = h ? (((meta.w >> 4) & 0x0F0F0F0Fu) | ((meta.z >> 2) & 0x30303030u)) : (meta.z & 0x3F3F3F3Fu);
}

// ------------------------------------------------------------------------------ helpers
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

__device__ __forceinline__ long long seg_stage_bytes(const GemvParams& P, int i) {
  return (long long)P.seg[i].tr * block_bytes(P.seg[i].w.type) * P.seg[i].w.G;
}

// CTA stage range balanced by bytes (segments differ in bytes per stage).
__device__ __forceinline__ void cta_stage_range(const GemvParams& P, int& s0, int& s1) {
  long long total = 0;
  for (int i = 0; i < P.nseg; ++i) total += (long long)P.seg[i].nstage * seg_stage_bytes(P, i);
  auto stage_at = [&](long long target) -> int {
    long long acc = 0;
    for (int i = 0; i < P.nseg; ++i) {
      const long long sb = seg_stage_bytes(P, i);
      const long long segb = (long long)P.seg[i].nstage * sb;
      if (target < acc + segb) return P.seg[i].stage0 + (int)((target - acc + sb - 1) / sb);
      acc += segb;
    }
    return P.nstages;
  };
  s0 = stage_at(total * (long long)blockIdx.x / gridDim.x);
  s1 = stage_at(total * (long long)(blockIdx.x + 1) / gridDim.x);
}

// Prologue item (unit u, part q): the 8 consecutive columns 256g + 128h + 32k + 16jh + 8(q%2) + i,
// k = q/2. A unit's 8 items sit in 8 consecutive lanes (LPR*8 and the thread count are multiples
// of 32), so the unit max is a 3-step shuffle.
__device__ __forceinline__ int item_col0(int item) {
  const int u = item >> 3, q = item & 7;
  const int g = u >> 2, uu = u & 3, h = uu >> 1, jh = uu & 1;
  return g * 256 + h * 128 + (q >> 1) * 32 + jh * 16 + (q & 1) * 8;
}

// Eight embedding-row values of a Q4_K row (bit-exact q4_decode order), from the device layout.
__device__ __forceinline__ void embed8_q4k(const QView& m, int row, int col0, float (&v)[8]) {
  const int G = m.G, g = col0 >> 8, e = col0 & 255;
  const int h = e >> 7, k6 = (e >> 5) & 3, j0 = e & 31, jh = j0 >> 4, jp0 = j0 & 15, u = 2 * h + jh;
  const uint4 meta = *reinterpret_cast<const uint4*>(m.base + row_plane_off(Q4K, G, row, 1, (size_t)g * 16));
  const uint2 nb = *reinterpret_cast<const uint2*>(
      m.base + row_plane_off(Q4K, G, row, 0, (size_t)(k6 >> 1) * 64 * G + (size_t)g * 64 + u * 16 + jp0));
  uint32_t scw, mnw;
  q4k_scale_words(meta, h, scw, mnw);
  const float d = h2f_bits(meta.x & 0xFFFFu), dm = h2f_bits(meta.x >> 16);
  const float sc = (float)((scw >> (8 * k6)) & 0xFF), mn = (float)((mnw >> (8 * k6)) & 0xFF);
  const float ds = __fmul_rn(d, sc), ms = __fmul_rn(dm, mn);
  const uint32_t w[2] = {nb.x, nb.y};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int q = (w[i >> 2] >> (8 * (i & 3) + (k6 & 1) * 4)) & 15;
    v[i] = __fsub_rn(__fmul_rn(ds, (float)q), ms);
  }
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = __ldcg(reinterpret_cast<const float4*>(p)), b = __ldcg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Prologue: residual + norm (or plain activations), digit planes and per-unit scalars into shared
// memory. One pass: every thread issues all of its loads first and keeps the values in registers,
// then the norm reduction, then the exact digit split (integer rounding done on the FMA pipe).
// MAXI bounds the prologue items per thread (8 columns each) the caller guarantees. A plain
// (XS_PLAIN) prologue may be split into calls over item blocks it_base, it_base + MAXI, ...;
// only the call with `last` ends with the barrier that publishes the planes. With GPRE the norm
// weights gm were loaded by the caller (gemv_load_gamma, before the dependency wait: they are
// constants of the model, not outputs of the preceding kernel).
template <int MAXI, bool GPRE>
__device__ __forceinline__ void gemv_prologue_core(const GemvParams& P, uint8_t* smem, const GemvSmem& L, int nthr_c,
                                                   int it_base, bool last, float (&gm)[MAXI][8]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint4* xplanes = reinterpret_cast<uint4*>(smem + L.xplanes);
  float* xscal = reinterpret_cast<float*>(smem + L.xscal);
  double* redd = reinterpret_cast<double*>(smem + L.redd);
  const int LPR = P.LPR, nitems = LPR * 8;
  int tok = 0;
  if (P.xmode == XS_EMBED) {
    tok = P.st->tok;
    if (tok < 0 || tok >= P.vocab) {
      if (tid == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_TOKEN);
      tok = 0;
    }
  }
  float v[MAXI][8];
  // ---- loads (all issued before any use, the norm weights included)
#pragma unroll
  for (int it = 0; it < MAXI; ++it) {
    const int item = tid + (it_base + it) * nthr_c;
    if (item < nitems) {
      const int col0 = item_col0(item);
      if (P.xmode == XS_PLAIN) {
        load8(P.x + col0, v[it]);
      } else if (P.xmode == XS_EMBED) {
        if (P.emb.type == Q4K) embed8_q4k(P.emb, tok, col0, v[it]);
        else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[it][i] = dequant_elem(P.emb, tok, col0 + i);
        }
      }
      if (P.xmode != XS_PLAIN && !GPRE) load8(P.gamma + col0, gm[it]);
      if (P.xmode == XS_NORM) {
        float hv[8], yv[8];
        load8(P.h_in + col0, hv);
        if (P.y_add) load8(P.y_add + col0, yv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[it][i] = P.y_add ? __fadd_rn(hv[i], yv[i]) : hv[i];
      }
    }
  }
  // ---- residual write-back and the norm scale (q4_rms q4.cu:39-46 / rmsfold kcpu4.c:123-139)
  if (P.xmode != XS_PLAIN) {
    double acc = 0.0;
    const bool wr = blockIdx.x == 0 && P.h_out;
#pragma unroll
    for (int it = 0; it < MAXI; ++it) {
      const int item = tid + (it_base + it) * nthr_c;
      if (item < nitems) {
        if (wr) {
          float4* ho = reinterpret_cast<float4*>(P.h_out + item_col0(item));
          ho[0] = make_float4(v[it][0], v[it][1], v[it][2], v[it][3]);
          ho[1] = make_float4(v[it][4], v[it][5], v[it][6], v[it][7]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = __dadd_rn(acc, __dmul_rn((double)v[it][i], (double)v[it][i]));
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) redd[warp] = acc;
    named_bar(KQ_BAR_PROLOGUE, nthr_c);
    if (tid == 0) KQ_TRACE_AT(P.trace_id, 6);
    double tot = 0.0;
    for (int w = 0; w < nthr_c / 32; ++w) tot += redd[w];
    const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / (double)P.C), P.eps)));
#pragma unroll
    for (int it = 0; it < MAXI; ++it) {
      const int item = tid + (it_base + it) * nthr_c;
      if (item < nitems) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[it][i] = __fmul_rn(__fmul_rn(v[it][i], s), gm[it][i]);
      }
    }
  }
  // ---- exact digit split per unit
  const float RND = 12582912.0f;   // 1.5 * 2^23: adding it rounds to an integer (RNE), |y| <= 128
#pragma unroll
  for (int it = 0; it < MAXI; ++it) {
    const int item = tid + (it_base + it) * nthr_c;
    if (item >= nitems) break;            // uniform across a warp
    const int u = item >> 3, q = item & 7, k = q >> 1, half = q & 1;
    float m = 0.f;
    int bad = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = fabsf(v[it][i]);
      bad |= !(a <= FLT_MAX);
      m = fmaxf(m, a);
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    int e = 0;
    if (!bad && m >= 0x1p-100f) {
      e = ((__float_as_int(m) >> 23) & 0xFF) - 127 - 6;   // m is normal here
      if (m > 127.f * pow2f(e)) ++e;
    }
    const float s1 = pow2f(e), s2 = pow2f(e - 7), i1 = pow2f(-e), i2 = pow2f(7 - e), i3 = pow2f(14 - e);
    // Every product below is by a power of two and exact (x1 s1 and x2 s2: small integers times
    // normal powers of two), or so small that the integer rounding gives RND either way, so the
    // fused forms equal the separate multiply and add.
    int dq[3][8];
    int S0 = 0, S1 = 0, S2 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = bad ? 0.f : v[it][i];
      const float t1 = __fmaf_rn(x, i1, RND);
      const float x1 = __fsub_rn(t1, RND);
      const float r1 = __fmaf_rn(-x1, s1, x);
      const float t2 = __fmaf_rn(r1, i2, RND);
      const float x2 = __fsub_rn(t2, RND);
      const float r2 = __fmaf_rn(-x2, s2, r1);
      const float t3 = __fmaf_rn(r2, i3, RND);
      dq[0][i] = __float_as_int(t1) - 0x4B400000;
      dq[1][i] = __float_as_int(t2) - 0x4B400000;
      dq[2][i] = __float_as_int(t3) - 0x4B400000;
      S0 += dq[0][i]; S1 += dq[1][i]; S2 += dq[2][i];
    }
    uint32_t w[3][2];   // the low bytes (two's complement digits), four per word
#pragma unroll
    for (int p = 0; p < 3; ++p)
#pragma unroll
      for (int j = 0; j < 2; ++j)
        w[p][j] = __byte_perm(__byte_perm((uint32_t)dq[p][4 * j], (uint32_t)dq[p][4 * j + 1], 0x0040),
                              __byte_perm((uint32_t)dq[p][4 * j + 2], (uint32_t)dq[p][4 * j + 3], 0x0040), 0x5410);
#pragma unroll
    for (int p = 0; p < 3; ++p)
      *reinterpret_cast<uint2*>(reinterpret_cast<uint32_t*>(&xplanes[(k * 3 + p) * LPR + u]) + half * 2) =
          make_uint2(w[p][0], w[p][1]);
    S0 += __shfl_xor_sync(0xffffffffu, S0, 1);
    S1 += __shfl_xor_sync(0xffffffffu, S1, 1);
    S2 += __shfl_xor_sync(0xffffffffu, S2, 1);
    if (half == 0) {
      xscal[(2 + k) * LPR + u] = (float)(S0 * 16384 + S1 * 128 + S2);
      reinterpret_cast<int*>(xscal)[(6 + k) * LPR + u] = 32 * S0;
      reinterpret_cast<int*>(xscal)[(10 + k) * LPR + u] = 32 * S1;
      reinterpret_cast<int*>(xscal)[(14 + k) * LPR + u] = 32 * S2;
    }
    if (q == 0) {
      xscal[0 * LPR + u] = pow2f(e - 14);
      xscal[1 * LPR + u] = bad ? __int_as_float(0x7fc00000) : 0.f;
    }
  }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 7);
  if (last) named_bar(KQ_BAR_PROLOGUE, nthr_c);
}

template <int MAXI = KQ_MAX_ITEMS>
__device__ __forceinline__ void gemv_prologue(const GemvParams& P, uint8_t* smem, const GemvSmem& L, int nthr_c,
                                              int it_base = 0, bool last = true) {
  float gm[MAXI][8];
  gemv_prologue_core<MAXI, false>(P, smem, L, nthr_c, it_base, last, gm);
}

// The norm weights of this thread's prologue items (item blocks from 0), for gemv_prologue_core
// with GPRE; nothing for a plain prologue.
template <int MAXI = KQ_MAX_ITEMS>
__device__ __forceinline__ void gemv_load_gamma(const GemvParams& P, int nthr_c, float (&gm)[MAXI][8]) {
  if (P.xmode == XS_PLAIN) return;
  const int nitems = P.LPR * 8;
#pragma unroll
  for (int it = 0; it < MAXI; ++it) {
    const int item = threadIdx.x + it * nthr_c;
    if (item < nitems) load8(P.gamma + item_col0(item), gm[it]);
  }
}

// Sum over the LPR threads of a row group of RPG per-thread partials. For LPR >= 32 the warp
// sums are combined across the row's warps through `red` (this stage's buffer) after a named
// barrier; for LPR < 32 the row group is a segment of a warp. Returns, in thread u == rr of the
// row group (rr < RPG), the total of row rr.
template <int RPG>
__device__ __forceinline__ float rows_reduce(const float (&p)[RPG], int u, int rg, int LPR, float* red, int bar0 = 1) {
  const int lane = threadIdx.x & 31;
  if (LPR < 32) {
    float mine = 0.f;
#pragma unroll
    for (int rr = 0; rr < RPG; ++rr) {
      float v = p[rr];
      for (int off = LPR >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (u == rr) mine = v;
    }
    return mine;
  }
  // reduce-scatter inside the warp: afterwards the lanes of block rr (32/RPG lanes) hold row rr
  float v;
  if (RPG == 1) {
    v = p[0];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  } else if (RPG == 2) {
    const bool up = lane & 16;
    v = (up ? p[RPG - 1] : p[0]) + __shfl_xor_sync(0xffffffffu, up ? p[0] : p[RPG - 1], 16);
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  } else {
    const bool up = lane & 16, mid = lane & 8;
    const float a0 = (up ? p[2 % RPG] : p[0]) + __shfl_xor_sync(0xffffffffu, up ? p[0] : p[2 % RPG], 16);
    const float a1 = (up ? p[3 % RPG] : p[1 % RPG]) + __shfl_xor_sync(0xffffffffu, up ? p[1 % RPG] : p[3 % RPG], 16);
    v = (mid ? a1 : a0) + __shfl_xor_sync(0xffffffffu, mid ? a0 : a1, 8);
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  }
  const int WPR = LPR >> 5, wr = u >> 5, span = 32 / RPG;
  // row held by this lane: RPG 4 -> lanes 0-7 row 0, 8-15 row 1, 16-23 row 2, 24-31 row 3
  const int myrow = RPG == 4 ? (((lane >> 4) << 1) | ((lane >> 3) & 1)) : lane / span;
  if ((lane % span) == 0) red[(rg * RPG + myrow) * WPR + wr] = v;
  if (WPR > 1) named_bar(bar0 + rg, LPR);
  else __syncwarp();
  float sum = 0.f;
  if (u < RPG)
    for (int w = 0; w < WPR; ++w) sum += red[(rg * RPG + u) * WPR + w];
  return sum;
}

// ------------------------------------------------------------------------------ consumer pieces
// Shared by k_gemv (one GEMV per launch) and the persistent decode kernel (one GEMV per phase).

// Per-thread consumer state of one GEMV.
struct GemvThread {
  int lane, rg, u, h, g, WPR;
  int bar0;          // named barrier of row group 0 of this lane
  int pos;           // the step's position (0 when out of range)
  bool kv_ok;        // the position lies inside the cache
  XS xs;
  float s3q;
  const float* rope_c;
  const float* rope_s;
  const uint4* xplanes;
  float* red;
  float bv;          // ARGMAX: best value / index seen by this thread
  int bi;
};

__device__ __forceinline__ void gemv_thread_init(const GemvParams& P, uint8_t* smem, const GemvSmem& L, int pos, GemvThread& T) {
  const int tid = threadIdx.x, LPR = P.LPR, lt = tid % (LPR * P.NRG);
  T.lane = tid / (LPR * P.NRG);
  T.rg = lt / LPR;
  T.u = lt % LPR;
  T.h = (T.u & 3) >> 1;
  T.g = T.u >> 2;
  T.WPR = LPR >= 32 ? LPR >> 5 : 1;
  T.bar0 = 1 + T.lane * P.NRG;
  T.kv_ok = pos >= 0 && pos < P.ctx;   // the host validates; never store outside the cache
  T.pos = T.kv_ok ? pos : 0;
  T.rope_c = reinterpret_cast<const float*>(smem + L.rope);
  T.rope_s = T.rope_c + KQ_MAX_HALF_HD;
  T.xplanes = reinterpret_cast<const uint4*>(smem + L.xplanes);
  T.red = reinterpret_cast<float*>(smem + L.red) + T.lane * 2 * 4 * P.NRG * T.WPR;   // RPG <= 4
  T.bv = -FLT_MAX;
  T.bi = 0x7fffffff;
}

// The rotary row of the step's rotary position into shared memory; the prologue's barriers
// publish it.
__device__ __forceinline__ void gemv_load_rope(const GemvParams& P, uint8_t* smem, const GemvSmem& L, const GemvThread& T) {
  const int tid = threadIdx.x;
  float* rc = reinterpret_cast<float*>(smem + L.rope);
  if (P.cos_t && tid < (P.hd >> 1)) {
    int rp = P.st ? P.st->rpos : 0;
    if (rp < 0 || rp >= P.ctx) rp = 0;   // the host validates
    rc[tid] = __ldcg(P.cos_t + (size_t)rp * (P.hd >> 1) + tid);
    rc[KQ_MAX_HALF_HD + tid] = __ldcg(P.sin_t + (size_t)rp * (P.hd >> 1) + tid);
  }
}

__device__ __forceinline__ void gemv_load_rope_at(const GemvParams& P, uint8_t* smem, const GemvSmem& L, int pos) {
  const int tid = threadIdx.x;
  float* rc = reinterpret_cast<float*>(smem + L.rope);
  if (P.cos_t && tid < (P.hd >> 1)) {
    rc[tid] = __ldcg(P.cos_t + (size_t)pos * (P.hd >> 1) + tid);
    rc[KQ_MAX_HALF_HD + tid] = __ldcg(P.sin_t + (size_t)pos * (P.hd >> 1) + tid);
  }
}

// After the prologue: this thread's per-unit activation scalars into registers.
__device__ __forceinline__ void gemv_load_xs(const GemvParams& P, uint8_t* smem, const GemvSmem& L, GemvThread& T) {
  const int LPR = P.LPR, u = T.u;
  const float* xscal = reinterpret_cast<const float*>(smem + L.xscal);
  T.xs.s3 = xscal[u];
  T.xs.poison = xscal[LPR + u];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    T.xs.xsf[k] = xscal[(2 + k) * LPR + u];
#pragma unroll
    for (int pl = 0; pl < 3; ++pl) T.xs.c[pl][k] = reinterpret_cast<const int*>(xscal)[(6 + 4 * pl + k) * LPR + u];
  }
  T.s3q = T.xs.s3 * 0.0625f;   // Q4_K sums carry a factor 16 (see q4k_group)
}

// Producer: the bytes and source of global stage s (whole 8-row tiles, one contiguous range).
__device__ __forceinline__ uint32_t gemv_stage_src(const GemvParams& P, int s, int& segi, const uint8_t** src) {
  while (s >= P.seg[segi].stage0 + P.seg[segi].nstage) ++segi;
  const QView& w = P.seg[segi].w;
  const int tr = P.seg[segi].tr;
  const int row0 = (s - P.seg[segi].stage0) * tr;
  const int rows = min(tr, w.R - row0);            // a multiple of 8 (whole tiles)
  *src = w.base + (size_t)(row0 >> 3) * tile_bytes(w.type, w.G);
  return (uint32_t)((size_t)(rows >> 3) * tile_bytes(w.type, w.G));
}

// Ring entries of the persistent kernel: up to P.tps consecutive stages of one segment.
// Returns the stage count of the entry starting at stage s (< n1); segi must be s's segment.
__device__ __forceinline__ int gemv_group(const GemvParams& P, int s, int n1, int segi) {
  const int seg_end = P.seg[segi].stage0 + P.seg[segi].nstage;
  return min(P.tps, min(n1, seg_end) - s);
}
__device__ __forceinline__ int gemv_group_count(const GemvParams& P, int n0, int n1) {
  int e = 0, segi = 0;
  for (int s = n0; s < n1; ++e) {
    while (s >= P.seg[segi].stage0 + P.seg[segi].nstage) ++segi;
    s += gemv_group(P, s, n1, segi);
  }
  return e;
}

// Epilogue of one finished row: global row `grow` of segment sg, its value, the value of row
// grow ^ 1 (pair epilogues: SwiGLU, rotary) and whether grow is the even row of its pair.
__device__ __forceinline__ void gemv_row_epilogue(const GemvParams& P, GemvThread& T, const Seg& sg, int grow, float fin,
                                                  float fin_odd, bool even) {
  const int epi = sg.epi;
  const int pos = T.pos;
  if (!T.kv_ok && (epi == EPI_ROPE_K || epi == EPI_V || epi == EPI_ROPE_Q)) atomicOr(P.err, KQ_DEV_ERR_BAD_POS);
  switch (epi) {
    case EPI_F32: sg.out_f[grow] = fin; break;
    case EPI_ARGMAX:
      sg.out_f[grow] = fin;
      if (fin > T.bv || (fin == T.bv && grow < T.bi)) { T.bv = fin; T.bi = grow; }
      break;
    case EPI_V: {
      const int kv = grow / P.hd, e = grow % P.hd;
      if (T.kv_ok) sg.out_h[((size_t)kv * P.ctx + pos) * P.hd + e] = __float2half_rn(fin);
    } break;
    case EPI_SWIGLU:
      if (even) sg.out_f[grow >> 1] = __fmul_rn(silu_f(fin), fin_odd);
      break;
    case EPI_ROPE_Q:
    case EPI_ROPE_K:
      if (even) {
        const int hh = grow / P.hd, i2 = (grow % P.hd) >> 1, half = P.hd >> 1;
        const float c = T.rope_c[i2], sn = T.rope_s[i2];
        const float o0 = __fsub_rn(__fmul_rn(fin, c), __fmul_rn(fin_odd, sn));
        const float o1v = __fadd_rn(__fmul_rn(fin, sn), __fmul_rn(fin_odd, c));
        if (epi == EPI_ROPE_Q) {
          sg.out_f[hh * P.hd + i2] = o0;
          sg.out_f[hh * P.hd + i2 + half] = o1v;
        } else if (T.kv_ok) {
          __half* dst = sg.out_h + ((size_t)hh * P.ctx + pos) * P.hd;
          dst[i2] = __float2half_rn(o0);
          dst[i2 + half] = __float2half_rn(o1v);
        }
      }
      break;
  }
}

// One stage (TR rows of segment segi starting at global stage s) from shared memory `buf`:
// load this thread's slice, release the slot (one arrive per warp on `empty_bar`; the warp whose
// arrival frees it calls on_free()), compute, reduce across the row group (reduction buffer
// `par` = 0/1 alternates between stages), epilogue.
struct NoHook {
  __device__ __forceinline__ void operator()() const {}
};
template <int TM, int RPG, class OnFree = NoHook>
__device__ __forceinline__ void gemv_stage(const GemvParams& P, GemvThread& T, int s, int segi, const uint8_t* buf,
                                           uint64_t* empty_bar, int par, const OnFree& on_free = OnFree()) {
  const int tid = threadIdx.x, rg = T.rg, u = T.u, h = T.h, g = T.g, G = P.G, NRG = P.NRG, LPR = P.LPR;
  const Seg& sg = P.seg[segi];
  const bool is_q4 = TM == TM_Q4K || (TM == TM_MIXED && sg.w.type == Q4K);
  const int row0 = (s - sg.stage0) * sg.tr;
  const int rows = min(sg.tr, sg.w.R - row0);
  const int type = is_q4 ? Q4K : Q6K;
  const size_t TB = tile_bytes(type, G);
  const size_t o1 = (size_t)8 * 128 * G;                                  // plane 1 in a tile
  const size_t o2 = o1 + (size_t)8 * (is_q4 ? 16 : 64) * G, o3 = o2 + (size_t)8 * 16 * G;
  // ---- load this thread's slice of its RPG rows, then free the stage
  uint32_t a[RPG][4], b[RPG][4], q[RPG][4];
  uint32_t m1[RPG];   // Q4_K: d | dmin << 16 ; Q6_K: four int8 scales
  uint32_t m2[RPG];   // Q4_K: 6-bit scales as 4 bytes ; Q6_K: fp16 d bits
  uint32_t m3[RPG];   // Q4_K: 6-bit mins as 4 bytes
#pragma unroll
  for (int rr = 0; rr < RPG; ++rr) {
    const int r = min(rg * RPG + rr, rows - 1);   // rows past a short last stage reuse a real one
    const uint8_t* tb = buf + (size_t)(r >> 3) * TB;
    const int r8 = r & 7;
    const uint8_t* p0 = tb + (size_t)r8 * 128 * G;
    const size_t sw = (size_t)r8 << 4;   // the plane-0 chunk swizzle (kq_qformat.cuh)
    const uint4 A = lds128(p0 + (((size_t)u * 16) ^ sw));
    const uint4 B = lds128(p0 + (((size_t)64 * G + u * 16) ^ sw));
    a[rr][0] = A.x; a[rr][1] = A.y; a[rr][2] = A.z; a[rr][3] = A.w;
    b[rr][0] = B.x; b[rr][1] = B.y; b[rr][2] = B.z; b[rr][3] = B.w;
    if (is_q4) {
      const uint4 M = lds128(tb + o1 + (size_t)r8 * 16 * G + q4_p1_swz(G, r8, (size_t)g * 16));
      q4k_scale_words(M, h, m2[rr], m3[rr]);
      m1[rr] = M.x;
      q[rr][0] = q[rr][1] = q[rr][2] = q[rr][3] = 0;
    } else {
      const uint4 H = lds128(tb + o1 + (size_t)r8 * 64 * G + q6_qh_swz(G, r8, (size_t)u * 16));
      q[rr][0] = H.x; q[rr][1] = H.y; q[rr][2] = H.z; q[rr][3] = H.w;
      m1[rr] = lds32(tb + o2 + (size_t)r8 * 16 * G + q4_p1_swz(G, r8, (size_t)u * 4));
      const size_t doff = ((size_t)r8 * G + g) * 2;
      const uint32_t dw = lds32(tb + o3 + (doff & ~(size_t)3));
      m2[rr] = (doff & 2) ? (dw >> 16) : (dw & 0xFFFFu);
      m3[rr] = 0;
    }
  }
  __syncwarp();
  if (empty_bar && (tid & 31) == 0) {   // null: the caller releases the slot after a later stage
    if (mbar_arrive_completes(empty_bar)) on_free();
  }
  // ---- compute: group by group, the digit planes shared by the RPG rows
  int Pi[RPG][3];
  float Q_[RPG];
#pragma unroll
  for (int rr = 0; rr < RPG; ++rr) { Pi[rr][0] = Pi[rr][1] = Pi[rr][2] = 0; Q_[rr] = 0.f; }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint4 xw[3];
#pragma unroll
    for (int pl = 0; pl < 3; ++pl) xw[pl] = T.xplanes[(k * 3 + pl) * LPR + u];
#pragma unroll
    for (int rr = 0; rr < RPG; ++rr) {
      if (is_q4) {
        q4k_group(k < 2 ? a[rr] : b[rr], k, m2[rr], xw, Pi[rr]);
        Q_[rr] = __fmaf_rn(byte_to_float_u(m3[rr], k), T.xs.xsf[k], Q_[rr]);
      } else {
        q6k_group(a[rr], b[rr], q[rr], k, m1[rr], xw, T.xs, Pi[rr]);
      }
    }
  }
  float part[RPG];
#pragma unroll
  for (int rr = 0; rr < RPG; ++rr) {
    const float Pf = planes_combine(Pi[rr]);
    if (is_q4) {
      const float d = h2f_bits(m1[rr] & 0xFFFFu), dm = h2f_bits(m1[rr] >> 16);
      part[rr] = __fadd_rn(__fsub_rn(__fmul_rn(T.s3q, __fmul_rn(d, Pf)), __fmul_rn(T.xs.s3, __fmul_rn(dm, Q_[rr]))), T.xs.poison);
    } else {
      part[rr] = __fadd_rn(__fmul_rn(T.xs.s3, __fmul_rn(h2f_bits(m2[rr]), Pf)), T.xs.poison);
    }
  }
  // ---- reduce across the row group; thread u == rr holds row rr
  const float fin = rows_reduce<RPG>(part, u, rg, LPR, T.red + par * RPG * NRG * T.WPR, T.bar0);
  // ---- epilogue
  const int epi = sg.epi;
  const bool pair_epi = epi == EPI_SWIGLU || epi == EPI_ROPE_Q || epi == EPI_ROPE_K;
  float fin_odd = 0.f;
  if (pair_epi) fin_odd = __shfl_down_sync(0xffffffffu, fin, 1);
  const int rloc = rg * RPG + u;
  if (u < RPG && rloc < rows) gemv_row_epilogue(P, T, sg, row0 + rloc, fin, fin_odd, (u & 1) == 0);
}

// ARGMAX epilogue across CTAs: each CTA's best (value, index) to P.part_val / P.part_idx, and
// the last CTA (ticket) merges them in CTA order (lowest index on ties), advances the step state
// and re-arms the ticket. Called by the consumer threads of every CTA.
// The CTA's best (value, index) over the n entries of bestv / besti to P.part_val / P.part_idx;
// the last CTA (ticket) merges all CTAs' pairs in CTA order (lowest index on ties), advances the
// step state and re-arms the ticket. Thread 0 of the CTA only.
__device__ __forceinline__ void gemv_argmax_merge(const GemvParams& P, const float* bestv, const int* besti, int n) {
  float v0 = -FLT_MAX; int i0 = 0x7fffffff;
  for (int r = 0; r < n; ++r)
    if (bestv[r] > v0 || (bestv[r] == v0 && besti[r] < i0)) { v0 = bestv[r]; i0 = besti[r]; }
  P.part_val[blockIdx.x] = v0;
  P.part_idx[blockIdx.x] = i0;
  __threadfence();
  const int t = atomicAdd(P.ticket, 1);
  if (t == (int)gridDim.x - 1) {
    __threadfence();
    float v1 = -FLT_MAX; int i1 = 0x7fffffff;
    for (int c = 0; c < (int)gridDim.x; ++c) {
      const float pv = *(volatile float*)&P.part_val[c];
      const int pi = *(volatile int*)&P.part_idx[c];
      if (pv > v1 || (pv == v1 && pi < i1)) { v1 = pv; i1 = pi; }
    }
    if (i1 == 0x7fffffff) i1 = 0;
    // advance the device-resident step state: the next step embeds this token at pos + 1
    DecodeState* st = P.st;
    st->next_tok = i1;
    if (P.out_ids && st->steps < P.out_cap) P.out_ids[st->steps] = i1;
    st->steps += 1;
    st->tok = i1;
    st->pos += 1;
    st->rpos = st->pos;          // the next step is a plain decode step
    st->tree_base = st->pos + 1;
    *P.ticket = 0;
  }
}

// ARGMAX epilogue across CTAs: each CTA's best (value, index) to P.part_val / P.part_idx, and
// the last CTA (ticket) merges them. Called by the consumer threads of every CTA.
template <int RPG>
__device__ __forceinline__ void gemv_argmax_tail(const GemvParams& P, uint8_t* smem, const GemvSmem& L, const GemvThread& T,
                                                 int nthr_c) {
  const int tid = threadIdx.x, NRG = P.NRG * P.nlanes;
  float* bestv = reinterpret_cast<float*>(smem + L.best);
  int* besti = reinterpret_cast<int*>(bestv + NRG * RPG);
  if (T.u < RPG) {
    const int r = (T.lane * P.NRG + T.rg) * RPG + T.u;
    bestv[r] = T.bv;
    besti[r] = T.bi;
  }
  named_bar(KQ_BAR_ARGMAX, nthr_c);
  if (tid == 0) gemv_argmax_merge(P, bestv, besti, NRG * RPG);
}

// The producer warp of a GEMV kernel (lane 0 works): this CTA's stages into the ring of nslots
// stage buffers at `stages`, full[slot] completing on the copy and s_stage[slot] naming the stage;
// the first P.prefetch stages are issued at once, the rest after the consumers' prologue (pro_bar)
// and as slots are released (empty). Fixed ranges: the nmine stages from s_begin. Claimed stages
// (P.dyn): stages come from a launch-wide counter, each claimed when the previous one is issued
// (the last 2 x grid stages only when a slot is free, so that no CTA holds a stage it cannot
// start yet), so a CTA that starts late (its SM still ran the previous kernel) takes fewer; the claim past
// the last stage becomes an end mark (s_stage = -1, full completed without a copy), and the last
// CTA to finish claiming re-arms the counters for the next launch. Stages claimed by one CTA
// increase, and each row is still computed by one CTA, so results do not depend on the claims.
// On a failed wait it drains its copies in flight (bounded).
__device__ __forceinline__ void gemv_producer(const GemvParams& P, uint8_t* stages, uint64_t* full, uint64_t* empty,
                                              uint64_t* pro_bar, int s_begin, int nmine, int* s_fail, int* s_issued,
                                              const int* s_done, int* s_stage) {
  if ((threadIdx.x & 31) != 0) return;
  const uint64_t pol = l2_evict_first_policy();
  int segi = 0;
  // claims ahead stop for the last two stages per CTA: those are claimed when a slot is free
  const int tail0 = P.nstages - 2 * (int)gridDim.x;
  int s_next = P.dyn ? atomicAdd(P.dyn, 1) : s_begin;   // < 0: none claimed ahead
  for (int i = 0; P.dyn || i < nmine; ++i) {
    const int slot = i % P.nslots;
    const uint32_t round = (uint32_t)(i / P.nslots);
    if (i == P.prefetch) {
      if (!mbar_wait(pro_bar, 0, P.err, KQ_DEV_ERR_WAIT_FULL)) { *s_fail = 1; break; }
    }
    if (i >= P.nslots) {
      if (!mbar_wait(&empty[slot], (round - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY)) { *s_fail = 1; break; }
    }
    if (*(volatile int*)s_fail) break;
    const int s = s_next >= 0 ? s_next : atomicAdd(P.dyn, 1);
    if (s >= P.nstages) {   // claimed past the end: the end mark
      *(volatile int*)&s_stage[slot] = -1;
      mbar_arrive(&full[slot]);
      break;
    }
    s_next = !P.dyn ? s + 1 : s < tail0 ? atomicAdd(P.dyn, 1) : -1;
    *(volatile int*)&s_stage[slot] = s;
    const uint8_t* src;
    const uint32_t bytes = gemv_stage_src(P, s, segi, &src);
    uint8_t* buf = stages + (size_t)slot * P.stage_bytes;
    mbar_arrive_expect_tx(&full[slot], bytes);
    bulk_g2s(buf, src, bytes, &full[slot], pol);
    *(volatile int*)s_issued = i + 1;
  }
  if (P.dyn) {
    __threadfence();   // this CTA's last claim is performed before it counts as done
    if (atomicAdd(P.dyn + 1, 1) == (int)gridDim.x - 1) {
      P.dyn[0] = 0;
      P.dyn[1] = 0;
    }
  }
  KQ_TRACE_AT(P.trace_id, 5);
  if (*(volatile int*)s_fail) {
    const int issued = *(volatile int*)s_issued;
    for (int j = *(volatile const int*)s_done; j < issued; ++j)
      if (!mbar_wait(&full[j % P.nslots], (uint32_t)(j / P.nslots) & 1, P.err, KQ_DEV_ERR_DRAIN)) break;
  }
}

// ------------------------------------------------------------------------------ the kernel
template <int TM, int RPG>
__global__ void __launch_bounds__(KQ_GEMV_MAX_THREADS, 1) k_gemv(const __grid_constant__ GemvParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int LPR = P.LPR, NRG = P.NRG;
  const int nthr_c = LPR * NRG;
  const int tid = threadIdx.x;
  const GemvSmem L = gemv_smem_layout(P.nslots, P.stage_bytes, LPR, NRG, RPG, nthr_c);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + P.nslots;
  __shared__ int s_fail, s_issued, s_done;
  __shared__ int s_stage[KQ_MAX_SLOTS];      // the stage in each ring slot
  __shared__ __align__(8) uint64_t pro_bar;   // completes when the consumers' prologue is done

  int s_begin, s_end;
  cta_stage_range(P, s_begin, s_end);
  const int nmine = s_end - s_begin;
  const int ncw = nthr_c >> 5;
  if (tid == 0) {
    for (int i = 0; i < P.nslots; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], ncw); }
    mbar_init(&pro_bar, 1);
    fence_mbar_init();
    s_fail = 0;
    s_issued = 0;
    s_done = 0;
  }
  __syncthreads();
  pdl_trigger();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 0);

  if (tid >= nthr_c) {
    // ---------------------------------------------------------------- producer warp
    if (tid < nthr_c + 32) gemv_producer(P, smem + L.stages, full, empty, &pro_bar, s_begin, nmine, &s_fail, &s_issued, &s_done, s_stage);
    pdl_wait();
    return;
  }

  // ------------------------------------------------------------------ consumers
  float gm[KQ_MAX_ITEMS][8];
  gemv_load_gamma(P, nthr_c, gm);   // constants: requested before the dependency wait
  // The step state (position, rotary position) and the rotary row are read before the
  // dependency wait too: the state is written before a step starts (by the host, or by the
  // previous step's output head), and a step's first kernel is launched with a full dependency
  // on that writer. (After the wait, the in-order warps stalled on the position's round trip
  // before issuing the prologue's loads.)
  GemvThread T;
  gemv_thread_init(P, smem, L, P.st ? P.st->pos : 0, T);
  gemv_load_rope(P, smem, L, T);
  pdl_wait();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 1);
  gemv_prologue_core<KQ_MAX_ITEMS, true>(P, smem, L, nthr_c, 0, true, gm);
  if (tid == 0) mbar_arrive(&pro_bar);
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 2);
  gemv_load_xs(P, smem, L, T);
  int segi = 0;
  for (int i = 0; P.dyn || i < nmine; ++i) {
    const int slot = i % P.nslots;
    const uint32_t round = (uint32_t)(i / P.nslots);
    if (!mbar_wait(&full[slot], round & 1, P.err, KQ_DEV_ERR_WAIT_FULL)) { s_fail = 1; break; }
    if (tid == 0 && i == 0) KQ_TRACE_AT(P.trace_id, 3);
    const int s = *(volatile int*)&s_stage[slot];
    if (s < 0) break;   // the producer's end mark
    while (s >= P.seg[segi].stage0 + P.seg[segi].nstage) ++segi;
    gemv_stage<TM, RPG>(P, T, s, segi, smem + L.stages + (size_t)slot * P.stage_bytes, &empty[slot], i & 1);
    if (tid == 0) *(volatile int*)&s_done = i + 1;
  }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 4);
  if (P.seg[0].epi == EPI_ARGMAX) gemv_argmax_tail<RPG>(P, smem, L, T, nthr_c);
}

}  // namespace kq
