// kq_gemv_mma.cuh -- single-token Q4_K / Q6_K GEMV with the multiply-adds on the tensor cores.
//
// The same job as k_gemv (kq_gemv.cuh): the decode step's q/k/v (Q4_K q, k and Q6_K v in one
// launch), o, gate/up and down GEMVs and config-0's matrix; the planner keeps long Q6_K-only
// launches (the output head) on k_gemv, whose dp4a consumer streams Q6_K faster once the
// prologue is amortised. k_gemv spends about three thread instructions per weight on dp4a
// digit-plane arithmetic; here one mma.sync.m16n8k32 (u8 weights x s8 activation digits, s32
// accumulation) does the work of 384 dp4a lanes.
//
//  * Weight stream: as in k_gemv (producer warp, 1-D bulk copies of whole 8-row tiles into an
//    mbarrier ring, stages fixed per CTA or claimed at run time), with Q4_K stages of 16 NB rows
//    and Q6_K stages of 8-32 rows (the segment's `tr`).
//  * Activations: the prologue (residual + fp64 RMS norm, embedding row or plain vector, exactly
//    as k_gemv's) splits x exactly into three int8 digit planes with one power-of-two scale per
//    256-column super-block, x = s3 (16384 x1 + 128 x2 + x3), stored per pair of 32-column
//    sub-blocks as MMA fragment bytes, plus the digit sums of every sub-block (the Q4_K dmin
//    term), the Q6_K "-32" table per 16-column half, and per super-block s3 and a NaN poison.
//  * Q4_K consumers: per pair of sub-blocks one ldmatrix.x4 brings 16 rows x 32 bytes of
//    nibbles (conflict-free thanks to the swizzled tile layout, kq_qformat.cuh) in A-fragment
//    order; the low and the high nibbles are two MMAs against the digit columns (planes 0-2 of
//    N = 8). Q6_K consumers (gm6_stage): one MMA per sub-block for the 8 rows of a tile, the
//    4-bit and 2-bit parts as the A rows. The int32 results are multiplied by the block scales
//    and summed per super-block in int32 (exact), then combined in fp32 with d (dmin) and the
//    activation scale, in a fixed order; the warps' row partials are summed in warp order. The
//    int32 sums are the exact dot products the dp4a form computes, so results agree with k_gemv
//    to fp32 rounding.
//  * Epilogues: those of k_gemv (gemv_row_epilogue), the argmax merge included.
#pragma once
#include "kq_gemv.cuh"

namespace kq {

// Launch shapes: NW consumer warps in NB groups; group b takes the rows 16 b .. 16 b + 15 of a
// stage of 16 NB rows, its NW / NB warps split the super-blocks.
constexpr int GM_MAX_WARPS = 16;
constexpr int GM_MAX_TR = 32;
constexpr int GM_MAXI = 6;                        // prologue items (8 columns) per thread at most

struct GmSmem {
  size_t stages, xb, xsf, xo, sbs, bars, red, redd, best, rope, total;
};
// xb: the activation digits as B fragments, per pair p of sub-blocks (2p, 2p+1) of a super-block
// and per plane L: 4 x 16 bytes, lane t's {b0, b1} of sub-block 2p then of 2p + 1.
// xo: the Q6_K offset terms, per sub-block 8 int32 for the 8 MMA columns (plane L, half jh) at
// 3 jh + L: -32 (-512 for the high-nibble sub-blocks) x the digit sum of the 16 columns.
__host__ __device__ inline GmSmem gm_smem_layout(int nslots, int stage_bytes, int C) {
  GmSmem s;
  size_t o = 0;
  s.stages = o; o += (size_t)nslots * stage_bytes;
  s.xb = o = gs_align(o, 16); o += (size_t)(C / 64) * 192;    // [pair][plane][t][16 bytes]
  s.xsf = o = gs_align(o, 16); o += (size_t)(C / 32) * 4;     // digit sums per sub-block
  s.xo = o = gs_align(o, 16); o += (size_t)(C / 32) * 32;     // [sub-block][column]
  s.sbs = o = gs_align(o, 16); o += (size_t)(C / 256) * 8;    // per super-block: s3, poison
  s.bars = o = gs_align(o, 8); o += (size_t)2 * nslots * 8;
  s.red = o = gs_align(o, 16); o += (size_t)2 * GM_MAX_WARPS * GM_MAX_TR * 4;
  s.redd = o = gs_align(o, 8); o += (size_t)GM_MAX_WARPS * 8;
  s.best = o = gs_align(o, 8); o += (size_t)GM_MAX_TR * 8;
  s.rope = o = gs_align(o, 16); o += (size_t)2 * KQ_MAX_HALF_HD * 4;
  s.total = gs_align(o, 128);
  return s;
}

__device__ __forceinline__ void gm_mma(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void gm_ldsm_x4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}

// Norm weights of this thread's prologue items (item i = columns 8i .. 8i + 7), before the
// dependency wait (model constants).
template <int NW, int MAXI>
__device__ __forceinline__ void gm_load_gamma(const GemvParams& P, float (&gm)[MAXI][8]) {
  if (P.xmode == XS_PLAIN) return;
#pragma unroll
  for (int it = 0; it < MAXI; ++it) {
    const int item = threadIdx.x + it * NW * 32;
    if (item < P.C / 8) load8(P.gamma + 8 * item, gm[it]);
  }
}

// Prologue: activations (plain, residual + norm, or embedding row) -> digit planes, sub-block
// digit sums and super-block scalars in shared memory. The digit split of every element is the
// one k_gemv's prologue performs (exact power-of-two steps), with the exponent taken over the
// element's 256-column super-block (the 32 items of one warp).
template <int NW, int MAXI>
__device__ __forceinline__ void gm_prologue(const GemvParams& P, uint8_t* smem, const GmSmem& L, const float (&gm)[MAXI][8],
                                            bool has6) {
  constexpr int NC = NW * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nitems = P.C / 8;
  uint8_t* xb = smem + L.xb;
  float* xsf = reinterpret_cast<float*>(smem + L.xsf);
  float* sbs = reinterpret_cast<float*>(smem + L.sbs);
  double* redd = reinterpret_cast<double*>(smem + L.redd);
  int tok = 0;
  if (P.xmode == XS_EMBED) {
    tok = P.st->tok;
    if (tok < 0 || tok >= P.vocab) {
      if (tid == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_TOKEN);
      tok = 0;
    }
  }
  float v[MAXI][8];
#pragma unroll
  for (int it = 0; it < MAXI; ++it) {
    const int item = tid + it * NC;
    if (item < nitems) {
      const int col0 = 8 * item;
      if (P.xmode == XS_PLAIN) {
        load8(P.x + col0, v[it]);
      } else if (P.xmode == XS_EMBED) {
        if (P.emb.type == Q4K) embed8_q4k(P.emb, tok, col0, v[it]);
        else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[it][i] = dequant_elem(P.emb, tok, col0 + i);
        }
      } else {
        float hv[8], yv[8];
        load8(P.h_in + col0, hv);
        if (P.y_add) load8(P.y_add + col0, yv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[it][i] = P.y_add ? __fadd_rn(hv[i], yv[i]) : hv[i];
      }
    }
  }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 6);
  if (P.xmode != XS_PLAIN) {
    // residual write-back and the norm (q4_rms q4.cu:39-46 / rmsfold kcpu4.c:123-139)
    double acc = 0.0;
    const bool wr = blockIdx.x == 0 && P.h_out;
#pragma unroll
    for (int it = 0; it < MAXI; ++it) {
      const int item = tid + it * NC;
      if (item < nitems) {
        if (wr) {
          float4* ho = reinterpret_cast<float4*>(P.h_out + 8 * item);
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
    if (tid == 0) KQ_TRACE_AT(P.trace_id, 7);
    named_bar(KQ_BAR_PROLOGUE, NC);
    if (tid == 0) KQ_TRACE_AT(P.trace_id, 8);
    double tot = 0.0;
    for (int w = 0; w < NW; ++w) tot += redd[w];
    const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / (double)P.C), P.eps)));
#pragma unroll
    for (int it = 0; it < MAXI; ++it) {
      const int item = tid + it * NC;
      if (item < nitems) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[it][i] = __fmul_rn(__fmul_rn(v[it][i], s), gm[it][i]);
      }
    }
  }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 9);
  // ---- exact digit split, one exponent per super-block (a warp's 32 items)
  const float RND = 12582912.0f;   // 1.5 * 2^23: adding it rounds to an integer (RNE), |y| <= 128
#pragma unroll
  for (int it = 0; it < MAXI; ++it) {
    const int item = tid + it * NC;
    if (item >= nitems) break;            // uniform across a warp (nitems is a multiple of 32)
    const int col0 = 8 * item, sbi = col0 >> 5, j0 = col0 & 31;
    float m = 0.f;
    int bad = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = fabsf(v[it][i]);
      bad |= !(a <= FLT_MAX);
      m = fmaxf(m, a);
    }
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    int e = 0;
    if (!bad && m >= 0x1p-100f) {
      e = ((__float_as_int(m) >> 23) & 0xFF) - 127 - 6;   // m is normal here
      if (m > 127.f * pow2f(e)) ++e;
    }
    const float s1 = pow2f(e), s2 = pow2f(e - 7), i1 = pow2f(-e), i2 = pow2f(7 - e), i3 = pow2f(14 - e);
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
    // B-fragment slots: bytes j0 .. j0 + 3 are word (b = j0 / 16) of lane t = (j0 % 16) / 4,
    // bytes j0 + 4 .. j0 + 7 the same word of lane t + 1; sub-block 2p + hi at 8 hi bytes in
    uint8_t* xq = xb + (size_t)(sbi >> 1) * 192 + (sbi & 1) * 8 + (j0 >> 4) * 4 + ((j0 & 15) >> 2) * 16;
#pragma unroll
    for (int p = 0; p < 3; ++p) {
      uint32_t w[2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
        w[j] = __byte_perm(__byte_perm((uint32_t)dq[p][4 * j], (uint32_t)dq[p][4 * j + 1], 0x0040),
                           __byte_perm((uint32_t)dq[p][4 * j + 2], (uint32_t)dq[p][4 * j + 3], 0x0040), 0x5410);
      *reinterpret_cast<uint32_t*>(xq + p * 64) = w[0];
      *reinterpret_cast<uint32_t*>(xq + p * 64 + 16) = w[1];
    }
    // digit sums of the 16-column halves (2 consecutive lanes), then of the sub-block (4 lanes)
    S0 += __shfl_xor_sync(0xffffffffu, S0, 1);
    S1 += __shfl_xor_sync(0xffffffffu, S1, 1);
    S2 += __shfl_xor_sync(0xffffffffu, S2, 1);
    if (has6 && (lane & 1) == 0) {
      // the Q6_K "-32" in the units of the sub-block's sums (16 for the high nibbles)
      const int f = (sbi & 3) >= 2 ? -512 : -32, jh = (j0 >> 4) * 3;
      int* xo = reinterpret_cast<int*>(smem + L.xo) + (size_t)sbi * 8;
      xo[jh] = f * S0;
      xo[jh + 1] = f * S1;
      xo[jh + 2] = f * S2;
      if (jh) { xo[6] = 0; xo[7] = 0; }
    }
    S0 += __shfl_xor_sync(0xffffffffu, S0, 2);
    S1 += __shfl_xor_sync(0xffffffffu, S1, 2);
    S2 += __shfl_xor_sync(0xffffffffu, S2, 2);
    if ((lane & 3) == 0) xsf[sbi] = (float)(S0 * 16384 + S1 * 128 + S2);
    if (tid == 0) KQ_TRACE_AT(P.trace_id, 10);
    if (lane == 0) {
      sbs[2 * (col0 >> 8)] = pow2f(e - 14);
      sbs[2 * (col0 >> 8) + 1] = bad ? __int_as_float(0x7fc00000) : 0.f;
    }
  }
  named_bar(KQ_BAR_PROLOGUE, NC);
}

// One stage (up to 16 NB rows of Q4_K segment segi, global stage s) from shared memory `buf`;
// finished rows go through gemv_row_epilogue in threads 0 .. rows-1.
template <int NW, int NB>
__device__ __forceinline__ void gm_stage(const GemvParams& P, GemvThread& T, int s, int segi, const uint8_t* buf,
                                         uint64_t* empty_bar, int par, uint8_t* smem, const GmSmem& L) {
  constexpr int TR = 16 * NB, NWG = NW / NB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t = lane & 3;
  const int blk = warp % NB, wg = warp / NB;
  const Seg& sg = P.seg[segi];
  const int G = P.G;
  const int row0 = (s - sg.stage0) * TR;
  const int rows = min(TR, sg.w.R - row0);            // a multiple of 8
  const int ntile = rows >> 3;
  const size_t TB = tile_bytes(Q4K, G), o1 = (size_t)8 * 128 * G;
  // tiles of this warp's 16-row block; a short stage reads its last tile again (rows unused)
  const int tA = min(2 * blk, ntile - 1), tB = min(2 * blk + 1, ntile - 1);
  // ldmatrix row of this lane: matrix mi = lane / 8 (tile mi & 1, 16-byte half mi >> 1), row lane % 8
  const int mi = lane >> 3, mr = lane & 7, jh = mi >> 1;
  const uint8_t* lrow = buf + (size_t)((mi & 1) ? tB : tA) * TB + (size_t)mr * 128 * G;
  const uint8_t* hdrA = buf + (size_t)tA * TB + o1 + (size_t)g8 * 16 * G;   // rows g8 and g8 + 8 of the block
  const uint8_t* hdrB = buf + (size_t)tB * TB + o1 + (size_t)g8 * 16 * G;
  const uint8_t* xb = smem + L.xb;
  const float* xsf = reinterpret_cast<const float*>(smem + L.xsf);
  const float* sbs = reinterpret_cast<const float*>(smem + L.sbs);
  const int sb0 = wg * G / NWG, sb1 = (wg + 1) * G / NWG;
  float acc = 0.f;   // lane t = 0: row g8 of the block; t = 1: row g8 + 8
  for (int sb = sb0; sb < sb1; ++sb) {
    const size_t ho = q4_p1_swz(G, g8, (size_t)sb * 16);
    const uint4 MA = lds128(hdrA + ho), MB = lds128(hdrB + ho);
    uint32_t scA[2], mnA[2], scB[2], mnB[2];
    q4k_scale_words(MA, 0, scA[0], mnA[0]);
    q4k_scale_words(MA, 1, scA[1], mnA[1]);
    q4k_scale_words(MB, 0, scB[0], mnB[0]);
    q4k_scale_words(MB, 1, scB[1], mnB[1]);
    // low- and high-nibble sums apart (the high nibbles are used in place: 16 q); per lane row g8
    // planes (2t, 2t+1), then row g8 + 8 planes (2t, 2t+1)
    int PL[4] = {0, 0, 0, 0}, PH[4] = {0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int c = p & 1, h = p >> 1, k = 2 * p;   // sub-blocks k (low nibbles), k + 1 (high)
      const size_t off = (size_t)c * 64 * G + (size_t)sb * 64 + h * 32 + jh * 16;
      uint32_t r[4];
      gm_ldsm_x4(lrow + p0_swz(mr, off), r);
      uint4 bx = make_uint4(0u, 0u, 0u, 0u);
      if (g8 < 3) bx = lds128(xb + ((size_t)(sb * 4 + p) * 3 + g8) * 64 + t * 16);
      const uint32_t al[4] = {r[0] & 0x0F0F0F0Fu, r[1] & 0x0F0F0F0Fu, r[2] & 0x0F0F0F0Fu, r[3] & 0x0F0F0F0Fu};
      const uint32_t ah[4] = {r[0] & 0xF0F0F0F0u, r[1] & 0xF0F0F0F0u, r[2] & 0xF0F0F0F0u, r[3] & 0xF0F0F0F0u};
      int dl[4], dh[4];
      gm_mma(dl, al, bx.x, bx.y);
      gm_mma(dh, ah, bx.z, bx.w);
      const uint32_t sel = 0x4440u + (uint32_t)(k & 3);
      const int sAl = (int)__byte_perm(scA[h], 0u, sel), sAh = (int)__byte_perm(scA[h], 0u, sel + 1);
      const int sBl = (int)__byte_perm(scB[h], 0u, sel), sBh = (int)__byte_perm(scB[h], 0u, sel + 1);
      PL[0] += sAl * dl[0]; PL[1] += sAl * dl[1]; PL[2] += sBl * dl[2]; PL[3] += sBl * dl[3];
      PH[0] += sAh * dh[0]; PH[1] += sAh * dh[1]; PH[2] += sBh * dh[2]; PH[3] += sBh * dh[3];
    }
    int Pa[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) Pa[i] = 16 * PL[i] + PH[i];   // every sum carries 16
    // lane t = 0 holds planes 0, 1 of both rows, lane t = 1 plane 2: row g8 is finished by t = 0,
    // row g8 + 8 by t = 1
    const int q2A = __shfl_down_sync(0xffffffffu, Pa[0], 1);
    const int q0B = __shfl_up_sync(0xffffffffu, Pa[2], 1);
    const int q1B = __shfl_up_sync(0xffffffffu, Pa[3], 1);
    if (t < 2) {
      const bool isB = t == 1;
      const int P3[3] = {isB ? q0B : Pa[0], isB ? q1B : Pa[1], isB ? Pa[2] : q2A};
      const float Pf = planes_combine(P3);
      const uint32_t dw = isB ? MB.x : MA.x;
      const float d = h2f_bits(dw & 0xFFFFu), dm = h2f_bits(dw >> 16);
      const uint32_t mn0 = isB ? mnB[0] : mnA[0], mn1 = isB ? mnB[1] : mnA[1];
      const float4 x0 = *reinterpret_cast<const float4*>(xsf + (size_t)sb * 8);
      const float4 x1 = *reinterpret_cast<const float4*>(xsf + (size_t)sb * 8 + 4);
      float Q = 0.f;
      Q = __fmaf_rn(byte_to_float_u(mn0, 0), x0.x, Q);
      Q = __fmaf_rn(byte_to_float_u(mn0, 1), x0.y, Q);
      Q = __fmaf_rn(byte_to_float_u(mn0, 2), x0.z, Q);
      Q = __fmaf_rn(byte_to_float_u(mn0, 3), x0.w, Q);
      Q = __fmaf_rn(byte_to_float_u(mn1, 0), x1.x, Q);
      Q = __fmaf_rn(byte_to_float_u(mn1, 1), x1.y, Q);
      Q = __fmaf_rn(byte_to_float_u(mn1, 2), x1.z, Q);
      Q = __fmaf_rn(byte_to_float_u(mn1, 3), x1.w, Q);
      const float2 sc = *reinterpret_cast<const float2*>(sbs + 2 * sb);   // s3, poison
      const float s3q = sc.x * 0.0625f;
      acc = __fadd_rn(acc, __fadd_rn(__fsub_rn(__fmul_rn(s3q, __fmul_rn(d, Pf)), __fmul_rn(sc.x, __fmul_rn(dm, Q))), sc.y));
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);   // this warp's reads of the stage are done
  float* red = reinterpret_cast<float*>(smem + L.red) + par * NW * GM_MAX_TR;
  if (t < 2) red[(16 * blk + g8 + 8 * t) * NWG + wg] = acc;
  named_bar(1, NW * 32);
  if (warp == 0) {
    float fin = 0.f;
    if (lane < TR)
      for (int w = 0; w < NWG; ++w) fin = __fadd_rn(fin, red[lane * NWG + w]);
    const float fin_odd = __shfl_down_sync(0xffffffffu, fin, 1);
    if (lane < rows) gemv_row_epilogue(P, T, sg, row0 + lane, fin, fin_odd, (lane & 1) == 0);
  }
}

// Byte k of w, sign-extended (prmt's sign-replicating selector: byte k, then three copies of its
// sign).
__device__ __forceinline__ int gm_sbyte(uint32_t w, int k) {
  const uint32_t sel = (uint32_t)k | ((uint32_t)(8 | k) * 0x1110u);
  uint32_t r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
  return (int)r;
}
__device__ __forceinline__ void gm6_mma(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c0, int c1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%12};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(0));
}

// One stage of a Q6_K segment: sg.tr / 8 tiles of 8 rows (nt); warp w takes tile w % nt and the
// super-blocks [wg G / NWG, (wg + 1) G / NWG), wg = w / nt, NWG = NW / nt.
// Per 32-column sub-block (h, k6) ONE mma.m16n8k32 does the 8 rows: A rows 0-7 are the rows'
// 4-bit parts (ql, low or high nibbles in place), A rows 8-15 the same rows' 2-bit parts (qh,
// bits 2 k6 in place), both read by ldmatrix from the swizzled tile; the B columns are the
// activation digit planes split by 16-column half (column 3 jh + L: plane L, zero outside half
// jh), because a Q6_K scale covers 16 columns; C carries the "-32" (the xo table). The lane
// holding D rows g8 / g8 + 8 thus has the 4-bit and the 2-bit sums of row g8 for two columns
// and combines them exactly (the 2-bit part shifted to weight 16); the scale of each (row, half)
// is applied in int32 and the planes are summed per super-block, then combined in fp32 with d
// and the activation scale, as k_gemv does.
template <int NW>
__device__ __forceinline__ void gm6_stage(const GemvParams& P, GemvThread& T, int s, int segi, const uint8_t* buf,
                                          uint64_t* empty_bar, int par, uint8_t* smem, const GmSmem& L) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t = lane & 3;
  const Seg& sg = P.seg[segi];
  const int G = P.G, tr = sg.tr, nt = tr >> 3, NWG = NW / nt;
  const int row0 = (s - sg.stage0) * tr;
  const int rows = min(tr, sg.w.R - row0);           // a multiple of 8
  const int tile = warp % nt, wg = warp / nt;
  // a short stage reads its last tile again (rows unused)
  const uint8_t* tb = buf + (size_t)min(tile, (rows >> 3) - 1) * tile_bytes(Q6K, G);
  const size_t o1 = (size_t)8 * 128 * G, o2 = o1 + (size_t)8 * 64 * G, o3 = o2 + (size_t)8 * 16 * G;
  // ldmatrix: matrix mi = lane / 8 is 16-byte chunk mi of the 64 bytes of (h, jh) = (mi / 2, mi % 2)
  const int mi = lane >> 3, mr = lane & 7;
  const uint8_t* lrow = tb + (size_t)mr * 128 * G;        // ql of tile row mr
  const uint8_t* qrow = tb + o1 + (size_t)mr * 64 * G;    // qh of tile row mr
  // B column g8 of this lane: plane g8 % 3 of half g8 / 3 (columns 6, 7 read real data, unused)
  const int bjh = g8 >= 3 ? 1 : 0, bpl = min(g8 - 3 * bjh, 2);
  const uint8_t* xa = smem + L.xb + bpl * 64 + t * 16 + bjh * 4;
  const int* xo = reinterpret_cast<const int*>(smem + L.xo) + 2 * t;
  const float* sbs = reinterpret_cast<const float*>(smem + L.sbs);
  // D columns 2t, 2t + 1 of this lane: halves ja, jb
  const bool ja = 2 * t >= 3, jb = 2 * t + 1 >= 3;
  const uint8_t* scrow = tb + o2 + (size_t)g8 * 16 * G;   // scales of row g8
  const uint8_t* drow = tb + o3 + (size_t)g8 * 2 * G;     // d of row g8
  const int sb0 = wg * G / NWG, sb1 = (wg + 1) * G / NWG;
  float acc = 0.f;   // lanes t = 0: row g8 of the tile
  for (int sb = sb0; sb < sb1; ++sb) {
    uint32_t q[4], r0[4], r1[4];
    gm_ldsm_x4(qrow + q6_qh_swz(G, mr, (size_t)sb * 64 + 16 * mi), q);
    gm_ldsm_x4(lrow + p0_swz(mr, (size_t)sb * 64 + 16 * mi), r0);                    // c = 0
    gm_ldsm_x4(lrow + p0_swz(mr, (size_t)64 * G + (size_t)sb * 64 + 16 * mi), r1);   // c = 1
    const uint4 S = lds128(scrow + q4_p1_swz(G, g8, (size_t)sb * 16));   // [u = 2h + jh][k6]
    const uint32_t wa0 = ja ? S.y : S.x, wa1 = ja ? S.w : S.z, wb0 = jb ? S.y : S.x, wb1 = jb ? S.w : S.z;
    int PL0 = 0, PL1 = 0, PH0 = 0, PH1 = 0;   // 4-bit-unit sums (PH: high nibbles, weight 16)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int k6 = 0; k6 < 4; ++k6) {
        const uint32_t* r = (k6 & 1) ? r1 : r0;
        const uint32_t m = (k6 >> 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu, mq = 0x03030303u << (2 * k6);
        const uint32_t a[4] = {r[2 * h] & m, q[2 * h] & mq, r[2 * h + 1] & m, q[2 * h + 1] & mq};
        const int sbi = sb * 8 + 4 * h + k6;
        const uint32_t av = lds32(xa + (size_t)(sbi >> 1) * 192 + (sbi & 1) * 8);
        const int2 cx = *reinterpret_cast<const int2*>(xo + (size_t)sbi * 8);
        int d[4];
        gm6_mma(d, a, bjh ? 0u : av, bjh ? av : 0u, cx.x, cx.y);
        const int sh = (k6 & 1) ? 2 : 4;                  // qh bits 2 k6 to weight 16 (x16 more: high)
        const int E0 = d[0] + (d[2] << sh), E1 = d[1] + (d[3] << sh);
        const int sa = gm_sbyte(h ? wa1 : wa0, k6), sc = gm_sbyte(h ? wb1 : wb0, k6);
        if (k6 >> 1) { PH0 += sa * E0; PH1 += sc * E1; }
        else { PL0 += sa * E0; PL1 += sc * E1; }
      }
    }
    // the high-nibble sums are exact multiples of 16
    const int Pa0 = PL0 + (PH0 >> 4), Pa1 = PL1 + (PH1 >> 4);   // columns 2t, 2t + 1
    // planes of row g8: column L (half 0) + column 3 + L (half 1), gathered in lane t = 0
    const int c2 = __shfl_down_sync(0xffffffffu, Pa0, 1), c3 = __shfl_down_sync(0xffffffffu, Pa1, 1);
    const int c4 = __shfl_down_sync(0xffffffffu, Pa0, 2), c5 = __shfl_down_sync(0xffffffffu, Pa1, 2);
    if (t == 0) {
      const int P3[3] = {Pa0 + c3, Pa1 + c4, c2 + c5};
      const float Pf = planes_combine(P3);
      const float d = h2f_bits(*reinterpret_cast<const uint16_t*>(drow + (size_t)sb * 2));
      const float2 sc = *reinterpret_cast<const float2*>(sbs + 2 * sb);   // s3, poison
      acc = __fadd_rn(acc, __fadd_rn(__fmul_rn(sc.x, __fmul_rn(d, Pf)), sc.y));
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);   // this warp's reads of the stage are done
  float* red = reinterpret_cast<float*>(smem + L.red) + par * NW * GM_MAX_TR;
  if (t == 0) red[(tile * 8 + g8) * NWG + wg] = acc;
  named_bar(1, NW * 32);
  if (warp == 0) {
    float fin = 0.f;
    if (lane < rows)
      for (int w = 0; w < NWG; ++w) fin = __fadd_rn(fin, red[lane * NWG + w]);
    const float fin_odd = __shfl_down_sync(0xffffffffu, fin, 1);
    if (lane < rows) gemv_row_epilogue(P, T, sg, row0 + lane, fin, fin_odd, (lane & 1) == 0);
  }
}

// NW consumer warps, NB 16-row blocks per Q4_K stage; MAXI prologue items per thread
// (C <= 8 * MAXI * 32 * NW columns); TY 1: every segment is Q4_K, 2: some are Q6_K (the Q4_K-only
// instances carry no Q6_K code). With NW = 16 the 17 warps leave 96 registers a thread (one SM
// sub-partition holds 5 of them), with NW = 12 128.
template <int NW, int NB, int MAXI, int TY>
__global__ void __launch_bounds__((NW + 1) * 32, 1) k_gemv_mma(const __grid_constant__ GemvParams P) {
  constexpr int NC = NW * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const GmSmem L = gm_smem_layout(P.nslots, P.stage_bytes, P.C);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + P.nslots;
  __shared__ int s_fail, s_issued, s_done;
  __shared__ int s_stage[KQ_MAX_SLOTS];   // the stage in each ring slot
  __shared__ __align__(8) uint64_t pro_bar;
  int s_begin, s_end;
  cta_stage_range(P, s_begin, s_end);
  const int nmine = s_end - s_begin;
  if (tid == 0) {
    for (int i = 0; i < P.nslots; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], NW); }
    mbar_init(&pro_bar, 1);
    fence_mbar_init();
    s_fail = 0;
    s_issued = 0;
    s_done = 0;
  }
  __syncthreads();
  pdl_trigger();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 0);
  if (tid >= NC) {
    gemv_producer(P, smem + L.stages, full, empty, &pro_bar, s_begin, nmine, &s_fail, &s_issued, &s_done, s_stage);
    pdl_wait();
    return;
  }
  // ---- consumers
  float gm[MAXI][8];
  gm_load_gamma<NW, MAXI>(P, gm);   // model constants: requested before the dependency wait
  GemvThread T;
  T.bv = -FLT_MAX;
  T.bi = 0x7fffffff;
  const int pos = P.st ? P.st->pos : 0;   // written before the step's first kernel starts
  T.kv_ok = pos >= 0 && pos < P.ctx;
  T.pos = T.kv_ok ? pos : 0;
  T.rope_c = reinterpret_cast<const float*>(smem + L.rope);
  T.rope_s = T.rope_c + KQ_MAX_HALF_HD;
  if (P.cos_t && tid < (P.hd >> 1)) {
    int rp = P.st ? P.st->rpos : 0;
    if (rp < 0 || rp >= P.ctx) rp = 0;   // the host validates
    float* rc = reinterpret_cast<float*>(smem + L.rope);
    rc[tid] = __ldcg(P.cos_t + (size_t)rp * (P.hd >> 1) + tid);
    rc[KQ_MAX_HALF_HD + tid] = __ldcg(P.sin_t + (size_t)rp * (P.hd >> 1) + tid);
  }
  pdl_wait();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 1);
  gm_prologue<NW, MAXI>(P, smem, L, gm, TY == 2);
  if (tid == 0) mbar_arrive(&pro_bar);
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 2);
  int segi = 0;
  for (int i = 0; P.dyn || i < nmine; ++i) {
    const int slot = i % P.nslots;
    const uint32_t round = (uint32_t)(i / P.nslots);
    if (!mbar_wait(&full[slot], round & 1, P.err, KQ_DEV_ERR_WAIT_FULL)) { s_fail = 1; break; }
    if (tid == 0 && i == 0) KQ_TRACE_AT(P.trace_id, 3);
    const int s = *(volatile int*)&s_stage[slot];
    if (s < 0) break;   // the producer's end mark
    while (s >= P.seg[segi].stage0 + P.seg[segi].nstage) ++segi;
    const uint8_t* buf = smem + L.stages + (size_t)slot * P.stage_bytes;
    if (TY == 1 || P.seg[segi].w.type == Q4K) gm_stage<NW, NB>(P, T, s, segi, buf, &empty[slot], i & 1, smem, L);
    else gm6_stage<NW>(P, T, s, segi, buf, &empty[slot], i & 1, smem, L);
    if (tid == 0) *(volatile int*)&s_done = i + 1;
  }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 4);
  if (P.seg[0].epi == EPI_ARGMAX) {
    float* bestv = reinterpret_cast<float*>(smem + L.best);
    int* besti = reinterpret_cast<int*>(bestv + GM_MAX_TR);
    if (tid < GM_MAX_TR) {   // the epilogue lanes of warp 0 (rows of a stage: at most GM_MAX_TR)
      bestv[tid] = T.bv;
      besti[tid] = T.bi;
    }
    named_bar(KQ_BAR_ARGMAX, NC);
    if (tid == 0) gemv_argmax_merge(P, bestv, besti, GM_MAX_TR);
  }
}

// The kernel instances the host picks from: (warps, row blocks, segment types) and the prologue
// width.
typedef void (*GmFn)(GemvParams);
template <int NW, int NB, int TY>
__host__ inline GmFn gm_fn_for(int C) {
  return C <= 2 * 8 * 32 * NW ? k_gemv_mma<NW, NB, 2, TY> : k_gemv_mma<NW, NB, (12288 + 8 * 32 * NW - 1) / (8 * 32 * NW), TY>;
}

}  // namespace kq
