// kq_gemv.cuh -- fused-dequant Q4_K / Q6_K GEMV for single-token decode on sm_100a.
//
// Replaces the reference's q4_gemv (scripts/kindi_q4/kindi/q4.cu:18-27), q4_embed (:28-32),
// q4_rms (:39-46) and q4_silu (:36-38), and the rope / K-V store of engine.py:260-267.
//
// Design:
//  * Persistent CTAs, one producer warp per CTA streaming runs of TR rows ("stages") of every
//    weight plane from HBM into a shared-memory ring with 1-D bulk copies (cp.async.bulk, L2
//    evict-first), completion tracked by mbarriers. The producer starts before
//    griddepcontrol.wait, so the weight stream of kernel N+1 overlaps the tail of kernel N.
//  * Activations stay in registers. Thread u of a row group owns the 64 columns of "unit"
//    (g, h, jh) (see kq_qformat.cuh) for every row. Its 64 fp32 activations are split exactly
//    into three int8 digit planes x = s1*x1 + s2*x2 + s3*x3 (s1 a power of two with
//    max|x| <= 127*s1, s2 = s1/128, s3 = s1/16384; residual <= s1/32768), so the dot products
//    with 4- and 6-bit weights are exact int32 dp4a sums per 16-element group; the groups are
//    combined with the block scales in fp32 and the row partials summed with a fixed warp-shuffle
//    tree, then across the row's warps in a fixed order.
//  * Fusions: the prologue does the residual add + fp64 RMS norm (q4_rms) or the embedding-row
//    dequantisation (q4_embed); the epilogue does the NeoX rotary + fp16 K/V store, the V store,
//    SwiGLU, or the output-head argmax (lowest index on ties, like k_argmax kindi.cu:637-661).
#pragma once
#include "kq_common.cuh"
#include "kq_qformat.cuh"
#include <cfloat>

namespace kq {

enum { EPI_F32 = 0, EPI_ROPE_Q = 1, EPI_ROPE_K = 2, EPI_V = 3, EPI_SWIGLU = 4, EPI_ARGMAX = 5 };
enum { XS_PLAIN = 0, XS_NORM = 1, XS_EMBED = 2 };
constexpr int KQ_MAX_SEG = 4;
constexpr int KQ_GEMV_MAX_THREADS = 416;   // 384 consumers + 1 producer warp

struct DecodeState {   // device-resident per-step state
  int tok;        // token processed by this step
  int pos;        // its position
  int next_tok;   // argmax written by the output head
  int steps;      // steps completed by the device-resident loop
};

struct Seg {
  QView w;
  int stage0, nstage;   // global stage range of this segment
  int epi;
  float* out_f;         // F32 / ROPE_Q / SWIGLU / ARGMAX (logits)
  __half* out_h;        // ROPE_K / V: this layer's cache [n_kv][ctx][hd]
};

struct GemvParams {
  Seg seg[KQ_MAX_SEG];
  int nseg, nstages;
  int C, G, TR, LPR, NRG, RPG;
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
};

// ------------------------------------------------------------------------------ activations
struct XL {
  uint32_t w[4][3][4];   // [group k][digit plane][word] int8 x 4
  float s3;
  float xsf[4];          // sum of the group's digits, 16384*S1 + 128*S2 + S3, as float
  int c0[4], c1[4];      // 32*S1 and 32*(128*S2 + S3): the "-32" of Q6_K, exact
  float poison;          // NaN if any activation of the unit was not finite
};

__device__ __forceinline__ float pow2f(int k) { return __int_as_float((k + 127) << 23); }

// v[k][j']: the unit's 64 activations, column 256g + 128h + 32k + 16jh + j'.
__device__ __forceinline__ void build_xl(const float (&v)[4][16], XL& xl) {
  float m = 0.f;
  bool bad = false;
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float a = fabsf(v[k][j]);
      bad |= !(a <= FLT_MAX);
      m = fmaxf(m, a);
    }
  int e = 0;
  if (!bad && m >= 0x1p-100f) {
    e = ilogbf(m) - 6;
    if (m > 127.f * pow2f(e)) ++e;
  }
  const float s1 = pow2f(e), s2 = pow2f(e - 7), i1 = pow2f(-e), i2 = pow2f(7 - e), i3 = pow2f(14 - e);
  xl.s3 = pow2f(e - 14);
  xl.poison = bad ? __int_as_float(0x7fc00000) : 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int S0 = 0, S1 = 0, S2 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float x = bad ? 0.f : v[k][4 * i + b];
        const float x1 = rintf(__fmul_rn(x, i1));
        const float r1 = __fsub_rn(x, __fmul_rn(x1, s1));
        const float x2 = rintf(__fmul_rn(r1, i2));
        const float r2 = __fsub_rn(r1, __fmul_rn(x2, s2));
        const float x3 = rintf(__fmul_rn(r2, i3));
        const int q1 = (int)x1, q2 = (int)x2, q3 = (int)x3;
        S0 += q1; S1 += q2; S2 += q3;
        w0 |= (uint32_t)(q1 & 0xFF) << (8 * b);
        w1 |= (uint32_t)(q2 & 0xFF) << (8 * b);
        w2 |= (uint32_t)(q3 & 0xFF) << (8 * b);
      }
      xl.w[k][0][i] = w0; xl.w[k][1][i] = w1; xl.w[k][2][i] = w2;
    }
    xl.xsf[k] = (float)(S0 * 16384 + S1 * 128 + S2);
    xl.c0[k] = 32 * S0;
    xl.c1[k] = 32 * (S1 * 128 + S2);
  }
}

__device__ __forceinline__ float byte_to_float_u(uint32_t w, int i) {
  return __fsub_rn(__int_as_float((int)__byte_perm(w, 0x4B000000u, (uint32_t)(i | 0x7440))), 8388608.f);
}

// Row partial of a Q4_K unit: A, B = nibble chunks of planes 0/1, meta = 16-byte block header.
__device__ __forceinline__ float row_q4k(const uint4 A, const uint4 B, const uint4 meta, int h, const XL& xl) {
  const uint32_t a[4] = {A.x, A.y, A.z, A.w}, b[4] = {B.x, B.y, B.z, B.w};
  float T[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int acc0 = 0, acc1 = 0, acc2 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t src = k < 2 ? a[i] : b[i];
      const int nib = (int)((k & 1) ? ((src >> 4) & 0x0F0F0F0Fu) : (src & 0x0F0F0F0Fu));
      acc0 = __dp4a(nib, (int)xl.w[k][0][i], acc0);
      acc1 = __dp4a(nib, (int)xl.w[k][1][i], acc1);
      acc2 = __dp4a(nib, (int)xl.w[k][2][i], acc2);
    }
    T[k] = (float)(acc0 * 16384 + acc1 * 128 + acc2);
  }
  // six-bit scales / mins of sub-blocks 4h .. 4h+3 as four bytes (q4kernels.h:17-18)
  const uint32_t sc_w = h ? ((meta.w & 0x0F0F0F0Fu) | ((meta.y >> 2) & 0x30303030u)) : (meta.y & 0x3F3F3F3Fu);
  const uint32_t mn_w = h ? (((meta.w >> 4) & 0x0F0F0F0Fu) | ((meta.z >> 2) & 0x30303030u)) : (meta.z & 0x3F3F3F3Fu);
  float P = __fmul_rn(byte_to_float_u(sc_w, 0), T[0]);
  float Q = __fmul_rn(byte_to_float_u(mn_w, 0), xl.xsf[0]);
#pragma unroll
  for (int k = 1; k < 4; ++k) {
    P = __fmaf_rn(byte_to_float_u(sc_w, k), T[k], P);
    Q = __fmaf_rn(byte_to_float_u(mn_w, k), xl.xsf[k], Q);
  }
  const float d = h2f_bits(meta.x & 0xFFFFu), dm = h2f_bits(meta.x >> 16);
  return __fadd_rn(__fmul_rn(xl.s3, __fsub_rn(__fmul_rn(d, P), __fmul_rn(dm, Q))), xl.poison);
}

// Row partial of a Q6_K unit: A, B = ql chunks (planes 0/1), H = qh chunk, scw = 4 int8
// scales (k = 0..3), dbits = fp16 d.
__device__ __forceinline__ float row_q6k(const uint4 A, const uint4 B, const uint4 H, uint32_t scw, uint32_t dbits,
                                         const XL& xl) {
  const uint32_t a[4] = {A.x, A.y, A.z, A.w}, b[4] = {B.x, B.y, B.z, B.w}, q[4] = {H.x, H.y, H.z, H.w};
  float F[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int acc0 = 0, acc1 = 0, acc2 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t src = (k & 1) ? b[i] : a[i];
      const uint32_t lo = (k >> 1) ? ((src >> 4) & 0x0F0F0F0Fu) : (src & 0x0F0F0F0Fu);
      const uint32_t hi = (k == 0) ? ((q[i] << 4) & 0x30303030u)
                        : (k == 1) ? ((q[i] << 2) & 0x30303030u)
                        : (k == 2) ? (q[i] & 0x30303030u)
                                   : ((q[i] >> 2) & 0x30303030u);
      const int q6 = (int)(lo | hi);
      acc0 = __dp4a(q6, (int)xl.w[k][0][i], acc0);
      acc1 = __dp4a(q6, (int)xl.w[k][1][i], acc1);
      acc2 = __dp4a(q6, (int)xl.w[k][2][i], acc2);
    }
    const int th = acc0 - xl.c0[k];
    const int tl = acc1 * 128 + acc2 - xl.c1[k];
    F[k] = __fadd_rn(__fmul_rn((float)th, 16384.f), (float)tl);
  }
  float P = __fmul_rn((float)(int)(int8_t)(scw & 0xFF), F[0]);
#pragma unroll
  for (int k = 1; k < 4; ++k) P = __fmaf_rn((float)(int)(int8_t)((scw >> (8 * k)) & 0xFF), F[k], P);
  const float d = h2f_bits(dbits);
  return __fadd_rn(__fmul_rn(xl.s3, __fmul_rn(d, P)), xl.poison);
}

// ------------------------------------------------------------------------------ the kernel
__device__ __forceinline__ size_t seg_stage_bytes(const QView& w, int TR) {
  return (size_t)TR * block_bytes(w.type) * w.G;
}

// Partial sum of a row across the LPR threads of a row group; the result is in thread u == 0.
// red: [NRG][WPR] floats for this stage parity.
__device__ __forceinline__ float row_reduce(float v, int u, int rg, int LPR, float* red) {
  if (LPR < 32) {
    for (int off = LPR >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int WPR = LPR >> 5, wr = u >> 5;
  if ((u & 31) == 0) red[rg * WPR + wr] = v;
  named_bar(1 + rg, LPR);
  float s = 0.f;
  if (u == 0)
    for (int w = 0; w < WPR; ++w) s += red[rg * WPR + w];
  return s;
}

__device__ __forceinline__ double row_reduce_d(double v, int u, int rg, int LPR, double* redd) {
  if (LPR < 32) {
    for (int off = LPR >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int WPR = LPR >> 5, wr = u >> 5;
  if ((u & 31) == 0) redd[rg * WPR + wr] = v;
  named_bar(1 + rg, LPR);
  double s = 0.0;
  for (int w = 0; w < WPR; ++w) s += redd[rg * WPR + w];
  named_bar(1 + rg, LPR);
  return s;
}

__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// Loads the unit's 64 activations into v (and the residual-updated h into hv for XS_NORM).
__device__ __forceinline__ void load_x(const GemvParams& P, int u_thr, int rg, int LPR, double* redd, float (&v)[4][16]) {
  const int g = u_thr >> 2, uu = u_thr & 3, h = uu >> 1, jh = uu & 1;
  const int col0 = g * 256 + h * 128 + jh * 16;
  if (P.xmode == XS_PLAIN) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4* src = reinterpret_cast<const float4*>(P.x + col0 + 32 * k);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 t = src[i];
        v[k][4 * i] = t.x; v[k][4 * i + 1] = t.y; v[k][4 * i + 2] = t.z; v[k][4 * i + 3] = t.w;
      }
    }
    return;
  }
  // residual stream value for this unit
  if (P.xmode == XS_EMBED) {
    int tok = P.st->tok;
    if (tok < 0 || tok >= P.vocab) {
      if (u_thr == 0 && rg == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_TOKEN);
      tok = 0;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < 16; ++j) v[k][j] = dequant_elem(P.emb, tok, col0 + 32 * k + j);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4* hs = reinterpret_cast<const float4*>(P.h_in + col0 + 32 * k);
      const float4* ys = reinterpret_cast<const float4*>(P.y_add + col0 + 32 * k);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = hs[i];
        float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
        if (P.y_add) b = ys[i];
        v[k][4 * i] = __fadd_rn(a.x, b.x); v[k][4 * i + 1] = __fadd_rn(a.y, b.y);
        v[k][4 * i + 2] = __fadd_rn(a.z, b.z); v[k][4 * i + 3] = __fadd_rn(a.w, b.w);
      }
    }
  }
  if (blockIdx.x == 0 && rg == 0 && P.h_out) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float4* ho = reinterpret_cast<float4*>(P.h_out + col0 + 32 * k);
#pragma unroll
      for (int i = 0; i < 4; ++i) ho[i] = make_float4(v[k][4 * i], v[k][4 * i + 1], v[k][4 * i + 2], v[k][4 * i + 3]);
    }
  }
  // fp64 sum of squares (q4_rms kindi q4.cu:39-46 / rmsfold kcpu4.c:123-139)
  double acc = 0.0;
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int j = 0; j < 16; ++j) acc = __dadd_rn(acc, __dmul_rn((double)v[k][j], (double)v[k][j]));
  const double tot = row_reduce_d(acc, u_thr, rg, LPR, redd);
  const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / (double)P.C), P.eps)));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float4* gs = reinterpret_cast<const float4*>(P.gamma + col0 + 32 * k);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 gm = gs[i];
      v[k][4 * i] = __fmul_rn(__fmul_rn(v[k][4 * i], s), gm.x);
      v[k][4 * i + 1] = __fmul_rn(__fmul_rn(v[k][4 * i + 1], s), gm.y);
      v[k][4 * i + 2] = __fmul_rn(__fmul_rn(v[k][4 * i + 2], s), gm.z);
      v[k][4 * i + 3] = __fmul_rn(__fmul_rn(v[k][4 * i + 3], s), gm.w);
    }
  }
}

// CTA stage range balanced by bytes (segments differ in bytes per stage).
__device__ __forceinline__ void cta_stage_range(const GemvParams& P, int& s0, int& s1) {
  long long total = 0;
  for (int i = 0; i < P.nseg; ++i) total += (long long)P.seg[i].nstage * (long long)seg_stage_bytes(P.seg[i].w, P.TR);
  auto stage_at = [&](long long target) -> int {
    long long acc = 0;
    for (int i = 0; i < P.nseg; ++i) {
      const long long sb = (long long)seg_stage_bytes(P.seg[i].w, P.TR);
      const long long segb = (long long)P.seg[i].nstage * sb;
      if (target < acc + segb) return P.seg[i].stage0 + (int)((target - acc + sb - 1) / sb);
      acc += segb;
    }
    return P.nstages;
  };
  s0 = stage_at(total * (long long)blockIdx.x / gridDim.x);
  s1 = stage_at(total * (long long)(blockIdx.x + 1) / gridDim.x);
}

__global__ void __launch_bounds__(KQ_GEMV_MAX_THREADS, 1) k_gemv(const __grid_constant__ GemvParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int nthr_c = P.LPR * P.NRG;
  const int tid = threadIdx.x;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)P.nslots * P.stage_bytes);
  uint64_t* empty = full + P.nslots;
  const int WPR = P.LPR >= 32 ? (P.LPR >> 5) : 1;
  float* red = reinterpret_cast<float*>(empty + P.nslots);            // [2][RPG][NRG][WPR]
  double* redd = reinterpret_cast<double*>(red + 2 * P.RPG * P.NRG * WPR + 2);  // [NRG][WPR]
  float* bestv = reinterpret_cast<float*>(redd + P.NRG * WPR);          // [NRG]
  int* besti = reinterpret_cast<int*>(bestv + P.NRG);                   // [NRG]
  __shared__ int s_fail, s_issued, s_done;

  int s_begin, s_end;
  cta_stage_range(P, s_begin, s_end);
  const int nmine = s_end - s_begin;
  const int ncw = (nthr_c + 31) >> 5;
  if (tid == 0) {
    for (int i = 0; i < P.nslots; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], ncw); }
    fence_mbar_init();
    s_fail = 0;
    s_issued = 0;
    s_done = 0;
  }
  __syncthreads();
  pdl_trigger();

  if (tid >= nthr_c) {
    // ---------------------------------------------------------------- producer warp
    if (tid == nthr_c) {
      const uint64_t pol = l2_evict_first_policy();
      int segi = 0;
      for (int i = 0; i < nmine; ++i) {
        const int slot = i % P.nslots;
        const uint32_t round = (uint32_t)(i / P.nslots);
        if (i >= P.nslots) {
          if (!mbar_wait(&empty[slot], (round - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY)) { s_fail = 1; break; }
        }
        if (*(volatile int*)&s_fail) break;
        const int s = s_begin + i;
        while (s >= P.seg[segi].stage0 + P.seg[segi].nstage) ++segi;
        const QView& w = P.seg[segi].w;
        const size_t row0 = (size_t)(s - P.seg[segi].stage0) * P.TR;
        uint8_t* buf = smem + (size_t)slot * P.stage_bytes;
        const uint32_t b0 = (uint32_t)(P.TR * plane_row_bytes(w.type, 0, w.G));
        const uint32_t b1 = (uint32_t)(P.TR * plane_row_bytes(w.type, 1, w.G));
        const uint32_t b2 = (uint32_t)(P.TR * plane_row_bytes(w.type, 2, w.G));
        const uint32_t b3 = (uint32_t)(P.TR * plane_row_bytes(w.type, 3, w.G));
        mbar_arrive_expect_tx(&full[slot], b0 + b1 + b2 + b3);
        bulk_g2s(buf, w.p0 + row0 * plane_row_bytes(w.type, 0, w.G), b0, &full[slot], pol);
        bulk_g2s(buf + b0, w.p1 + row0 * plane_row_bytes(w.type, 1, w.G), b1, &full[slot], pol);
        if (b2) bulk_g2s(buf + b0 + b1, w.p2 + row0 * plane_row_bytes(w.type, 2, w.G), b2, &full[slot], pol);
        if (b3) bulk_g2s(buf + b0 + b1 + b2, w.p3 + row0 * plane_row_bytes(w.type, 3, w.G), b3, &full[slot], pol);
        *(volatile int*)&s_issued = i + 1;
      }
      // failure path only: wait (bounded) for the copies still in flight before the CTA can exit
      if (*(volatile int*)&s_fail) {
        const int issued = *(volatile int*)&s_issued;
        for (int j = *(volatile int*)&s_done; j < issued; ++j)
          if (!mbar_wait(&full[j % P.nslots], (uint32_t)(j / P.nslots) & 1, P.err, KQ_DEV_ERR_DRAIN)) break;
      }
    }
    pdl_wait();
    return;
  }

  // ------------------------------------------------------------------ consumers
  pdl_wait();
  const int rg = tid / P.LPR, u_thr = tid % P.LPR;
  const int h = (u_thr & 3) >> 1;
  const int g = u_thr >> 2;
  XL xl;
  {
    float v[4][16];
    load_x(P, u_thr, rg, P.LPR, redd, v);
    build_xl(v, xl);
  }
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  int segi = 0;
  const int G = P.G;
  for (int i = 0; i < nmine; ++i) {
    const int slot = i % P.nslots;
    const uint32_t round = (uint32_t)(i / P.nslots);
    if (!mbar_wait(&full[slot], round & 1, P.err, KQ_DEV_ERR_WAIT_FULL)) { s_fail = 1; break; }
    const int s = s_begin + i;
    while (s >= P.seg[segi].stage0 + P.seg[segi].nstage) ++segi;
    const Seg& sg = P.seg[segi];
    const uint8_t* buf = smem + (size_t)slot * P.stage_bytes;
    const int type = sg.w.type;
    float part[8];
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      if (rr >= P.RPG) break;
      const int r = rg * P.RPG + rr;   // row within the stage
      const uint8_t* p0 = buf + (size_t)r * 128 * G;
      const uint4 A = lds128(p0 + u_thr * 16);
      const uint4 B = lds128(p0 + (size_t)64 * G + u_thr * 16);
      const size_t b0 = (size_t)P.TR * 128 * G;
      if (type == Q4K) {
        const uint4 meta = lds128(buf + b0 + ((size_t)r * G + g) * 16);
        part[rr] = row_q4k(A, B, meta, h, xl);
      } else {
        const size_t b1 = (size_t)P.TR * 64 * G, b2 = (size_t)P.TR * 16 * G;
        const uint4 H = lds128(buf + b0 + (size_t)r * 64 * G + u_thr * 16);
        const uint32_t scw = lds32(buf + b0 + b1 + (size_t)r * 16 * G + u_thr * 4);
        const size_t doff = ((size_t)r * G + g) * 2;
        const uint32_t dw = lds32(buf + b0 + b1 + b2 + (doff & ~(size_t)3));
        part[rr] = row_q6k(A, B, H, scw, (doff & 2) ? (dw >> 16) : (dw & 0xFFFFu), xl);
      }
    }
    __syncwarp();
    if ((tid & 31) == 0) mbar_arrive(&empty[slot]);
    if (tid == 0) *(volatile int*)&s_done = i + 1;
    // reduce + epilogue
    float* redb = red + (i & 1) * P.RPG * P.NRG * WPR;
    float fin[8];
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      if (rr >= P.RPG) break;
      fin[rr] = row_reduce(part[rr], u_thr, rg, P.LPR, redb + rr * P.NRG * WPR);
    }
    if (u_thr == 0) {
      const int grow0 = (s - sg.stage0) * P.TR + rg * P.RPG;
      int pos = P.st ? P.st->pos : 0;
      const bool kv_ok = pos >= 0 && pos < P.ctx;   // the host validates; never store outside the cache
      if (!kv_ok && (sg.epi == EPI_ROPE_K || sg.epi == EPI_V || sg.epi == EPI_ROPE_Q)) {
        atomicOr(P.err, KQ_DEV_ERR_BAD_POS);
        pos = 0;
      }
      for (int rr = 0; rr < P.RPG; ++rr) {
        const int grow = grow0 + rr;
        const float val = fin[rr];
        switch (sg.epi) {
          case EPI_F32: sg.out_f[grow] = val; break;
          case EPI_ARGMAX:
            sg.out_f[grow] = val;
            if (val > bv || (val == bv && grow < bi)) { bv = val; bi = grow; }
            break;
          case EPI_V: {
            const int kv = grow / P.hd, e = grow % P.hd;
            if (kv_ok) sg.out_h[((size_t)kv * P.ctx + pos) * P.hd + e] = __float2half_rn(val);
          } break;
          case EPI_SWIGLU:
            if ((rr & 1) == 1) sg.out_f[grow >> 1] = __fmul_rn(silu_f(fin[rr - 1]), val);
            break;
          case EPI_ROPE_Q:
          case EPI_ROPE_K:
            if ((rr & 1) == 1) {
              const int hh = grow / P.hd, i2 = (grow % P.hd) >> 1, half = P.hd >> 1;
              const float a = fin[rr - 1], b = val;
              const float c = P.cos_t[(size_t)pos * half + i2], sn = P.sin_t[(size_t)pos * half + i2];
              const float o0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
              const float o1 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
              if (sg.epi == EPI_ROPE_Q) {
                sg.out_f[hh * P.hd + i2] = o0;
                sg.out_f[hh * P.hd + i2 + half] = o1;
              } else if (kv_ok) {
                __half* dst = sg.out_h + ((size_t)hh * P.ctx + pos) * P.hd;
                dst[i2] = __float2half_rn(o0);
                dst[i2 + half] = __float2half_rn(o1);
              }
            }
            break;
        }
      }
    }
  }
  // ------------------------------------------------------------------ argmax across CTAs
  if (P.seg[0].epi == EPI_ARGMAX) {
    if (u_thr == 0) { bestv[rg] = bv; besti[rg] = bi; }
    named_bar(15, nthr_c);
    if (tid == 0) {
      float v0 = -FLT_MAX; int i0 = 0x7fffffff;
      for (int r = 0; r < P.NRG; ++r)
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
        *P.ticket = 0;
      }
    }
  }
}

}  // namespace kq
