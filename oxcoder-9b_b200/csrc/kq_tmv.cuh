// kq_tmv.cuh -- single-token Q4_K / Q6_K GEMV on the 5th-generation tensor cores (tcgen05.mma
// kind::i8, A in tensor memory), for the decode step's per-layer projections.
//
// Replaces, for the q/k/v, o, gate/up and down projections of one token, the reference's
// q4_gemv (scripts/kindi_q4/kindi/q4.cu:18-27) with the same fusions as the CUDA-core k_gemv:
// residual + RMS norm prologue (q4_rms q4.cu:39-46), rotary + fp16 K/V store, V store, SwiGLU
// (q4_silu q4.cu:36-38) or a plain fp32 output.
//
// Arithmetic. The activation vector of each 256-column super-block is split exactly into three
// int8 digit planes, x = s3 * (16384 x1 + 128 x2 + x3) (s3 a power of two per super-block). The
// weights enter the MMA as their raw unsigned digits: Q4_K low nibbles as bytes q (w & 0x0F0F0F0F),
// high nibbles in place as 16 q (w & 0xF0F0F0F0), Q6_K as the 6-bit q. One MMA per 32-column
// group (K = 32, M = 128 rows, N = 8): its B operand is the group's three planes (rows 0-2 of the
// 8-row B tile; the other rows are don't-care, read from whatever follows in shared memory), so
// D columns 0-2 are the exact int32 dot products of the
// group's weight digits with each plane (for Q6_K, whose scale blocks are 16 columns, the B tile
// holds the first 16 columns' planes in rows 0-2 and the last 16's in rows 3-5, zero elsewhere).
// The thread owning the row then applies the integer sub-block scales in int32 (exact: |sum| <
// 2.5e8), combines the planes in fp32 and adds the d / dmin terms as k_gemv does.
//
// Work split ("stream-K"): the units (128-row tile t, super-block g), ordered t-major, are cut into
// one contiguous run per CTA (one CTA per SM, all resident). A CTA streams its run without a break
// at tile boundaries; a tile it covers whole gets its epilogue at once, the (at most two) tiles it
// shares with neighbours leave an fp32 partial and the last contributor (ticket) sums the partials
// in CTA order and runs the epilogue, so the result does not depend on timing. Warp roles:
//   warps 0-7   thread (row r = 32 (warp & 3) + lane, half hh = warp >> 2 of the super-block):
//               prologue (activation digits -> B tiles), then per unit its A digits to tensor
//               memory and the read-back of the previous unit's D; tile flushes and epilogues
//   warp 8      raw loader: lane 0 issues one bulk copy per unit from the matrix's unit-major copy
//               (see below)
//   warp 9      TMEM allocation (512 columns: A digits of two units in [0, 128), two D regions of
//               8 groups x 8 columns at 128 and 256); lane 0 issues the 8 MMAs of each unit
// Every wait is bounded; on a timeout the CTA records the error, skips the remaining work (every
// thread still takes the same barriers) and drains before it exits.
//
// Unit-major weight copy. In the kq tile layout a unit's bytes are 512 pieces of 16-64 B (each
// row's chunks of the super-block, rows 2 KB apart), which the copy engines move at ~16 GB/s per
// SM. Each matrix the decode step multiplies therefore also keeps a second copy (HBM holds both
// easily: the decode weights are ~4 GB of 180) in which every unit is stored exactly as its
// shared-memory stage image, so one 18-27 KB bulk copy moves it:
//   Q4_K (18432 B): [0, 8192) nibble chunk c = 0 as 128 rows x 64 B, [8192, 16384) c = 1, the 16-byte
//                   chunks of row r at position j ^ ((r >> 1) & 3) (conflict-free 16-byte reads by 8
//                   consecutive rows); [16384, 18432) block headers, 16 B per row
//   Q6_K (26880 B): [0, 16384) ql as above, [16384, 24576) qh (64 B per row, same chunk order),
//                   [24576, 26624) scales (16 B per row), [26624, 26880) d (2 B per row)
// Rows past the matrix are zero. k_tv_repack builds it from the tile layout.
#pragma once
#include "kq_common.cuh"
#include "kq_qformat.cuh"
#include "kq_gemv.cuh"
#include "kq_tmm.cuh"

namespace kq {

constexpr int TV_ROWS = 128;
constexpr int TV_DQ_WARPS = 8;                                    // A-digit writers
constexpr int TV_RO_WARPS = 4;                                    // D read-back, prologue, epilogues
constexpr int TV_LD_WARP = TV_DQ_WARPS + TV_RO_WARPS;             // raw loader
constexpr int TV_MMA_WARP = TV_LD_WARP + 1;                       // TMEM allocation, MMA issue
constexpr int TV_THREADS = (TV_MMA_WARP + 1) * 32;
constexpr int TV_AS = 4;                                          // A slots (64 columns each)
constexpr int TV_DS = 4;                                          // D slots (64 columns each)
constexpr int TV_HS = TV_AS + TV_DS;                              // header slots
constexpr int TV_RS = 5;                                          // raw unit stages
constexpr int TV_MAX_G = 48;                                      // super-blocks per row, at most
constexpr int TV_MAX_SEG = 3;
constexpr int TV_MAX_TILES = 4096;                                // row tiles per launch, at most
constexpr uint32_t TV_TMEM_COLS = 512;
constexpr int TV_MMA_N = 8;                                       // D columns per group (the MMA's N)
constexpr int TV_B_Q4 = 96, TV_B_Q6 = 144;                        // B bytes per 32-column group
constexpr int TV_B_PAD = 320;                                     // the 16-row B tile's don't-care rows
// Offsets inside a unit's stage image (see the unit-major copy above).
constexpr int TV_ST_C1 = 8192, TV_ST_HDR = 16384, TV_ST_QH = 16384, TV_ST_SC = 24576, TV_ST_D = 26624;
constexpr uint32_t TV_UNIT_Q4 = 18432, TV_UNIT_Q6 = 26880;
constexpr size_t TV_RAW_BYTES = TV_UNIT_Q6;                        // one ring stage (a multiple of 128 B)

// Dynamic shared memory, identical on host (sizing) and device: raw ring, s3[G], X32[G][8],
// C16[G][16] (int4), red[128], per-unit row headers hdr[TV_HS][128] (Q4_K block header / Q6_K
// scale words) and hdrd[TV_HS][128] (Q6_K d), the Q4_K-layout B tiles (if any Q4_K segment), the
// Q6_K-layout B tiles (if any Q6_K segment).
struct TvSmem {
  size_t s3, x32, c16, red, hdr, hdrd, bq4, bq6, total;
};
// (offsets from the 1024-byte aligned start; the launch adds 1024 bytes of alignment slack)
__host__ __device__ inline TvSmem tv_smem(int G, bool has_q4, bool has_q6) {
  TvSmem L;
  size_t o = (size_t)TV_RS * TV_RAW_BYTES;
  L.s3 = o; o += (size_t)G * 4;
  o = (o + 15) & ~(size_t)15;
  L.x32 = o; o += (size_t)G * 8 * 4;
  o = (o + 15) & ~(size_t)15;
  L.c16 = o; o += (size_t)G * 16 * 16;
  L.red = o; o += (size_t)TV_ROWS * 4;
  o = (o + 15) & ~(size_t)15;
  L.hdr = o; o += (size_t)TV_HS * TV_ROWS * 16;
  L.hdrd = o; o += (size_t)TV_HS * TV_ROWS * 4;
  L.bq4 = o; if (has_q4) o += (size_t)G * 8 * TV_B_Q4 + TV_B_PAD;
  o = (o + 15) & ~(size_t)15;
  L.bq6 = o; if (has_q6) o += (size_t)G * 8 * TV_B_Q6 + TV_B_PAD;
  L.total = ((o + 127) & ~(size_t)127) + 1024;
  return L;
}

struct TvSeg {
  QView w;              // w.tv: the unit-major copy
  int tile0;            // first row tile of this segment
  int epi;
  float* out_f;
  __half* out_h;
};

struct TmvParams {
  TvSeg seg[TV_MAX_SEG];
  int nseg, ntiles, G;
  int has_q4, has_q6;
  int smem;             // dynamic shared memory bytes (tv_smem(G, has_q4, has_q6).total)
  int xmode;            // XS_PLAIN or XS_NORM
  const float* x;
  const float* h_in;
  const float* y_add;
  const float* gamma;
  float* h_out;
  float eps;
  DecodeState* st;
  const float* cos_t;
  const float* sin_t;
  int hd, ctx;
  float* part;          // partials of shared tiles [gridDim.x][2][128]
  int* ticket;          // [ntiles], zero between launches
  int* err;
};

// Instruction descriptor, kind::i8: s32 D (2 at bit 4), A unsigned (0 at bit 7), B signed (1 at
// bit 10), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t tc_idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Shared-memory descriptor of an 8-row B tile, K-major without swizzle: 16-byte rows per K half
// (rows contiguous), the second K half `lbo` bytes after the first; the stride between 8-row
// groups (unused at N = 8) set to 128. Version 1 at bit 46, layout 0.
__device__ __forceinline__ uint64_t tv_bdesc(uint32_t saddr, uint32_t lbo) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) |
         ((uint64_t)1 << 46);
}
// D[tmem] = A[tmem] * B[smem desc]^T, kind::i8 (u8 x s8 -> s32), no accumulation.
__device__ __forceinline__ void tc_mma_i8_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, 0, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
// 4 / 8 consecutive 32-bit columns of this thread's TMEM lane; not waited (tc_wait_ld).
__device__ __forceinline__ void tc_ld4_nw(uint32_t taddr, int (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tc_ld8_nw(uint32_t taddr, int (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 consecutive 32-bit columns of this thread's TMEM lane; not waited (tc_wait_ld).
__device__ __forceinline__ void tc_ld32_nw(uint32_t taddr, int (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,"
      "%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

// Byte offset of 16-byte chunk j (0..3) of row r in a part of 64-byte rows of a stage image.
__host__ __device__ __forceinline__ int tv_sw64(int r, int j) { return r * 64 + 16 * (j ^ ((r >> 1) & 3)); }

// kq tile layout -> unit-major copy: one thread per (unit, row).
__global__ void __launch_bounds__(256) k_tv_repack(const QView w, uint8_t* tv) {
  const int G = w.G, ntiles = (w.R + TV_ROWS - 1) / TV_ROWS;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)ntiles * G * TV_ROWS) return;
  const int r = (int)(i % TV_ROWS);
  const long long unit = i / TV_ROWS;
  const int g = (int)(unit % G), t = (int)(unit / G), row = t * TV_ROWS + r;
  const bool ok = row < w.R, q4 = w.type == Q4K;
  uint8_t* dst = tv + (size_t)unit * (q4 ? TV_UNIT_Q4 : TV_UNIT_Q6);
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  auto ld16 = [&](int plane, size_t off) -> uint4 {
    return ok ? *reinterpret_cast<const uint4*>(w.base + row_plane_off(w.type, G, row, plane, off)) : z;
  };
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(dst + c * TV_ST_C1 + tv_sw64(r, j)) = ld16(0, (size_t)c * 64 * G + (size_t)g * 64 + 16 * j);
  if (q4) {
    *reinterpret_cast<uint4*>(dst + TV_ST_HDR + 16 * r) = ld16(1, (size_t)g * 16);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(dst + TV_ST_QH + tv_sw64(r, j)) = ld16(1, (size_t)g * 64 + 16 * j);
    *reinterpret_cast<uint4*>(dst + TV_ST_SC + 16 * r) = ld16(2, (size_t)g * 16);
    *reinterpret_cast<uint16_t*>(dst + TV_ST_D + 2 * r) =
        ok ? *reinterpret_cast<const uint16_t*>(w.base + row_plane_off(Q6K, G, row, 3, (size_t)g * 2)) : (uint16_t)0;
  }
}

// Unsigned byte k of w (the signed one is sbyte in kq_gemv.cuh).
__device__ __forceinline__ int tv_ubyte(uint32_t w, int k) { return (int)__byte_perm(w, 0, 0x4440u | (uint32_t)k); }

// Unit range of CTA c of n over U units, and the CTA that holds unit u.
__host__ __device__ inline long long tv_unit0(int c, int n, long long U) { return (long long)c * U / n; }
__host__ __device__ inline int tv_cta_of(long long u, int n, long long U) { return (int)(((u + 1) * n - 1) / U); }

// Prologue (warps 0-7): the activations of all G super-blocks as int8 digit planes in the MMA's B
// tiles (the Q4_K and / or the Q6_K layout, as the launch's segments need), and the per-super-block
// / per-group scalars: s3 (the digit unit), X32 (the digit sum of each 32-column group as a float,
// for the Q4_K min term) and C16 (32 x the digit sums of each 16 columns, for the Q6_K "-32").
// XS_NORM: residual add and RMS norm over all C columns first (q4_rms q4.cu:39-46; fp64 sum of
// squares), CTA 0 writing the residual sum to h_out. The digit split is k_gemv's, per super-block:
// s1 = 2^e with max |x| <= 127 s1, s2 = s1 / 128, s3 = s1 / 16384.
// Run by the NT threads tid = 0 .. NT - 1 of warps whose first is warp w0 (named barrier 2).
template <int NT>
__device__ __forceinline__ void tv_prologue(const TmvParams& P, uint8_t* sm, const TvSmem& L, double* redd, int tid) {
  const int lane = tid & 31, warp = tid >> 5;
  const int C = 256 * P.G;
  float ns = 1.f;
  if (P.xmode == XS_NORM) {
    double acc = 0.0;
    const bool wr = blockIdx.x == 0 && P.h_out;
    for (int c0 = 8 * tid; c0 < C; c0 += 8 * NT) {
      float hv[8], yv[8];
      load8(P.h_in + c0, hv);
      if (P.y_add) {
        load8(P.y_add + c0, yv);
#pragma unroll
        for (int i = 0; i < 8; ++i) hv[i] = __fadd_rn(hv[i], yv[i]);
      }
      if (wr) {
        float4* ho = reinterpret_cast<float4*>(P.h_out + c0);
        ho[0] = make_float4(hv[0], hv[1], hv[2], hv[3]);
        ho[1] = make_float4(hv[4], hv[5], hv[6], hv[7]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = __dadd_rn(acc, __dmul_rn((double)hv[i], (double)hv[i]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) redd[warp] = acc;
    named_bar(2, NT);
    double tot = 0.0;
    for (int w = 0; w < NT / 32; ++w) tot += redd[w];
    ns = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / (double)C), P.eps)));
  }
  uint8_t* bq4 = sm + L.bq4;
  uint8_t* bq6 = sm + L.bq6;
  float* s3a = reinterpret_cast<float*>(sm + L.s3);
  float* x32 = reinterpret_cast<float*>(sm + L.x32);
  int4* c16 = reinterpret_cast<int4*>(sm + L.c16);
  const float RND = 12582912.0f;   // 1.5 * 2^23: adding it rounds to an integer (RNE), |y| <= 128
  // chunk q = 8 columns; a warp holds one super-block (q >> 5 is warp-uniform)
  for (int q = tid; q < 32 * P.G; q += NT) {
    const int kb = q >> 5, j = q & 31, c0 = 256 * kb + 8 * j;
    float v[8];
    if (P.xmode == XS_NORM) {
      float hv[8], yv[8], gm[8];
      load8(P.h_in + c0, hv);
      load8(P.gamma + c0, gm);
      if (P.y_add) load8(P.y_add + c0, yv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(P.y_add ? __fadd_rn(hv[i], yv[i]) : hv[i], ns), gm[i]);
    } else {
      load8(P.x + c0, v);
    }
    float mx = 0.f;
    int bad = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = fabsf(v[i]);
      bad |= !(a <= FLT_MAX);
      mx = fmaxf(mx, a);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    int e = 0;
    if (!bad && mx >= 0x1p-100f) {
      e = ((__float_as_int(mx) >> 23) & 0xFF) - 127 - 6;   // mx is normal here
      if (mx > 127.f * pow2f(e)) ++e;
    }
    const float s1 = pow2f(e), s2 = pow2f(e - 7), i1 = pow2f(-e), i2 = pow2f(7 - e), i3 = pow2f(14 - e);
    uint32_t wv[3][2] = {{0, 0}, {0, 0}, {0, 0}};
    int S0 = 0, S1 = 0, S2 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = bad ? 0.f : v[i];
      const float t1 = __fadd_rn(__fmul_rn(x, i1), RND);
      const float x1 = __fsub_rn(t1, RND);
      const float r1 = __fsub_rn(x, __fmul_rn(x1, s1));
      const float t2 = __fadd_rn(__fmul_rn(r1, i2), RND);
      const float x2 = __fsub_rn(t2, RND);
      const float r2 = __fsub_rn(r1, __fmul_rn(x2, s2));
      const float t3 = __fadd_rn(__fmul_rn(r2, i3), RND);
      const int q1 = __float_as_int(t1) - 0x4B400000, q2 = __float_as_int(t2) - 0x4B400000,
                q3 = __float_as_int(t3) - 0x4B400000;
      S0 += q1; S1 += q2; S2 += q3;
      wv[0][i >> 2] |= (uint32_t)(q1 & 0xFF) << (8 * (i & 3));
      wv[1][i >> 2] |= (uint32_t)(q2 & 0xFF) << (8 * (i & 3));
      wv[2][i >> 2] |= (uint32_t)(q3 & 0xFF) << (8 * (i & 3));
    }
    // B tile of group gi = j >> 2 (32 columns); this chunk is its 8 columns 8p .. 8p + 7
    const int gi = j >> 2, p = j & 3;
    if (P.has_q4) {
      // [K half][plane][16 B]: rows 0-2 of the tile are the planes, the K halves 48 B apart
      uint8_t* b = bq4 + (size_t)(kb * 8 + gi) * TV_B_Q4 + 48 * (p >> 1) + 8 * (p & 1);
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) *reinterpret_cast<uint2*>(b + 16 * pl) = make_uint2(wv[pl][0], wv[pl][1]);
    }
    if (P.has_q6) {
      // [first 16 columns' planes][48 zero bytes][last 16 columns' planes]: the tile at +0 has rows
      // (a0 a1 a2 0 0 0 ..) in K half 0 and the one at +48 (0 0 0 b0 b1 b2 ..) in K half 1
      uint8_t* gb = bq6 + (size_t)(kb * 8 + gi) * TV_B_Q6;
      uint8_t* b = gb + ((p >> 1) ? 96 : 0) + 8 * (p & 1);
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) *reinterpret_cast<uint2*>(b + 16 * pl) = make_uint2(wv[pl][0], wv[pl][1]);
      if (p == 0) {
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(gb + 48) = z;
        *reinterpret_cast<uint4*>(gb + 64) = z;
        *reinterpret_cast<uint4*>(gb + 80) = z;
      }
    }
    S0 += __shfl_xor_sync(0xffffffffu, S0, 1);
    S1 += __shfl_xor_sync(0xffffffffu, S1, 1);
    S2 += __shfl_xor_sync(0xffffffffu, S2, 1);
    if (P.has_q6 && (j & 1) == 0) c16[kb * 16 + (j >> 1)] = make_int4(32 * S0, 32 * S1, 32 * S2, 0);
    S0 += __shfl_xor_sync(0xffffffffu, S0, 2);
    S1 += __shfl_xor_sync(0xffffffffu, S1, 2);
    S2 += __shfl_xor_sync(0xffffffffu, S2, 2);
    if (P.has_q4 && (j & 3) == 0) x32[kb * 8 + gi] = (float)(S0 * 16384 + S1 * 128 + S2);
    if (j == 0) s3a[kb] = bad ? __int_as_float(0x7fc00000) : pow2f(e - 14);
  }
}

// Epilogue of row lrow of segment S (value v; vo = the value of row lrow ^ 1), as k_gemv's.
__device__ __forceinline__ void tv_epilogue(const TmvParams& P, const TvSeg& S, int lrow, float v, float vo) {
  const int epi = S.epi;
  if (epi == EPI_F32) {
    S.out_f[lrow] = v;
    return;
  }
  int pos = P.st ? P.st->pos : 0;
  const bool kv_ok = pos >= 0 && pos < P.ctx;   // the host validates; never store outside the cache
  if (!kv_ok) {
    pos = 0;
    if (epi == EPI_ROPE_K || epi == EPI_V || epi == EPI_ROPE_Q) atomicOr(P.err, KQ_DEV_ERR_BAD_POS);
  }
  switch (epi) {
    case EPI_V: {
      const int kv = lrow / P.hd, e = lrow % P.hd;
      if (kv_ok) S.out_h[((size_t)kv * P.ctx + pos) * P.hd + e] = __float2half_rn(v);
    } break;
    case EPI_SWIGLU:
      if ((lrow & 1) == 0) S.out_f[lrow >> 1] = __fmul_rn(silu_f(v), vo);
      break;
    case EPI_ROPE_Q:
    case EPI_ROPE_K:
      if ((lrow & 1) == 0) {
        int rp = P.st ? P.st->rpos : 0;
        if (rp < 0 || rp >= P.ctx) rp = 0;   // the host validates
        const int hh = lrow / P.hd, i2 = (lrow % P.hd) >> 1, half = P.hd >> 1;
        const float c = __ldg(P.cos_t + (size_t)rp * half + i2), sn = __ldg(P.sin_t + (size_t)rp * half + i2);
        const float o0 = __fsub_rn(__fmul_rn(v, c), __fmul_rn(vo, sn));
        const float o1 = __fadd_rn(__fmul_rn(v, sn), __fmul_rn(vo, c));
        if (epi == EPI_ROPE_Q) {
          S.out_f[hh * P.hd + i2] = o0;
          S.out_f[hh * P.hd + i2 + half] = o1;
        } else if (kv_ok) {
          __half* dst = S.out_h + ((size_t)hh * P.ctx + pos) * P.hd;
          dst[i2] = __float2half_rn(o0);
          dst[i2 + half] = __float2half_rn(o1);
        }
      }
      break;
  }
}

// Bounded wait of the roles off the MMA thread's critical path: between probes the thread sleeps
// `ns`, so waiting warps leave the issue slots of their SM sub-partition to the MMA thread (which
// shares one with them). Gives up after TM_WAIT_NS, or at once when another role flagged a failure.
__device__ __forceinline__ bool tv_wait(uint64_t* bar, uint32_t parity, int* err, int bit, volatile int* abort_f, unsigned ns) {
  if (mbar_test_wait(bar, parity)) return true;
  uint64_t t0 = 0;
  for (uint32_t it = 0; it < KQ_WAIT_LIMIT; ++it) {
    __nanosleep(ns);
    if (mbar_test_wait(bar, parity)) return true;
    if ((it & 63) == 63) {
      if (*abort_f) return false;
      const uint64_t now = tm_clock_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > TM_WAIT_NS) break;
    }
  }
  atomicOr(err, bit);
  *abort_f = 1;
  return false;
}

// Bounded wait that ignores the abort flag: the final drain of the CTA's own MMAs, which finish
// on their own.
__device__ __forceinline__ void tv_drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint64_t t0 = tm_clock_ns();
  for (uint32_t it = 0; it < KQ_WAIT_LIMIT; ++it) {
    if (mbar_try_wait(bar, parity)) return;
    if ((it & 255) == 255 && tm_clock_ns() - t0 > TM_WAIT_NS) break;
  }
  atomicOr(err, KQ_DEV_ERR_DRAIN);
}

__global__ void __launch_bounds__(TV_THREADS, 1) k_tmv(const __grid_constant__ TmvParams P) {
  extern __shared__ __align__(128) uint8_t tv_sm[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tv_sm) + 1023) & ~(uintptr_t)1023);
  const TvSmem L = tv_smem(P.G, P.has_q4 != 0, P.has_q6 != 0);
  uint8_t* raw_ring = sm;
  uint4* hdr = reinterpret_cast<uint4*>(sm + L.hdr);         // [TV_HS][128]
  uint32_t* hdrd = reinterpret_cast<uint32_t*>(sm + L.hdrd);  // [TV_HS][128]
  // mdone[k % TV_AS]: the MMAs of unit k have completed (A slot free for unit k + TV_AS, D slot
  // ready for the read-back); d_free[k % TV_DS]: the read-back of unit k has its D and header
  static_assert(TV_AS == TV_DS, "one completion barrier per unit serves the A and the D slot");
  __shared__ __align__(8) uint64_t raw_full[TV_RS], raw_empty[TV_RS], a_full[TV_AS], mdone[TV_AS], d_free[TV_DS],
      h_full[TV_HS], b_ready, mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort, s_last;
  __shared__ double s_redd[TV_DQ_WARPS + TV_RO_WARPS];
  volatile int* abort_f = &s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = P.G, nct = (int)gridDim.x, cta = (int)blockIdx.x;
  const long long U = (long long)P.ntiles * G;
  const long long u0 = tv_unit0(cta, nct, U);
  const int n = (int)(tv_unit0(cta + 1, nct, U) - u0);
  auto seg_of = [&](int t) -> int {
    int si = 0;
    while (si + 1 < P.nseg && t >= P.seg[si + 1].tile0) ++si;
    return si;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < TV_RS; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], TV_DQ_WARPS); }
    for (int i = 0; i < TV_AS; ++i) { mbar_init(&a_full[i], TV_DQ_WARPS); mbar_init(&mdone[i], 1); }
    for (int i = 0; i < TV_DS; ++i) mbar_init(&d_free[i], TV_RO_WARPS);
    for (int i = 0; i < TV_HS; ++i) mbar_init(&h_full[i], 1);
    mbar_init(&b_ready, 1);
    mbar_init(&mma_done, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == TV_MMA_WARP) {
    tmem_alloc(&s_tmem, TV_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  pdl_trigger();
  if (threadIdx.x == 0) KQ_TRACE_AT(0, 10);

  if (warp == TV_LD_WARP) {
    // ---------------- raw loader (lane 0): one bulk copy per unit from the unit-major copy; the
    // weights do not depend on the previous kernel (no PDL wait)
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int k = 0;
      for (; k < n; ++k) {
        const int slot = k % TV_RS;
        if (k >= TV_RS && !tv_wait(&raw_empty[slot], (uint32_t)((k / TV_RS) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f, 64))
          break;
        const long long u = u0 + k;
        const int t = (int)(u / G), g = (int)(u % G);
        const TvSeg& S = P.seg[seg_of(t)];
        const uint32_t ub = S.w.type == Q4K ? TV_UNIT_Q4 : TV_UNIT_Q6;
        mbar_arrive_expect_tx(&raw_full[slot], ub);
        bulk_g2s(raw_ring + (size_t)slot * TV_RAW_BYTES, S.w.tv + ((size_t)(t - S.tile0) * G + g) * ub, ub, &raw_full[slot], pol);
      }
      // drain: the copies into the last stages have landed before the CTA exits
      for (int j = k - TV_RS < 0 ? 0 : k - TV_RS; j < k; ++j)
        tm_wait(&raw_full[j % TV_RS], (uint32_t)(j / TV_RS) & 1, P.err, KQ_DEV_ERR_DRAIN, abort_f);
    }
    __syncwarp();
  } else if (warp == TV_MMA_WARP) {
    // ---------------- MMA issue (one thread): unit k reads A slot k % TV_AS (columns 64 (k % TV_AS))
    // and writes D slot k % TV_DS (columns 256 + 64 (k % TV_DS), group gi at 8 gi)
    if (lane == 0) {
      const uint32_t idesc = tc_idesc_i8(TV_ROWS, TV_MMA_N);
      const uint32_t bq4 = smem_u32(sm + L.bq4), bq6 = smem_u32(sm + L.bq6);
      if (tm_wait(&b_ready, 0, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f)) {
        for (int k = 0; k < n; ++k) {
          // a_full implies both slots are free: its writers waited for the MMAs and the read-back
          // of unit k - TV_AS (one wait here; each mbarrier wait costs this thread ~200 cycles)
          const int as = k % TV_AS, ds = k % TV_DS;
          if (!tm_wait(&a_full[as], (uint32_t)(k / TV_AS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f)) break;
          KQ_TRACE_AT(k, 4);
          // hands the header slot of unit k (written before the writers' a_full arrivals, acquired
          // above) on to the read-back warps
          mbar_arrive(&h_full[k % TV_HS]);
          // (no tcgen05 fence here: the writers' tcgen05.wait::st before their arrival orders their
          // tensor-memory stores before these MMAs, as CUTLASS's transform-to-MMA pipeline does; a
          // fence::after_thread_sync per unit serialised each unit's MMAs behind the previous ones)
          const long long u = u0 + k;
          const int t = (int)(u / G), g = (int)(u % G);
          const bool q4 = P.seg[seg_of(t)].w.type == Q4K;
          const uint32_t bst = q4 ? TV_B_Q4 : TV_B_Q6, bb = (q4 ? bq4 : bq6) + (uint32_t)g * 8u * bst;
          const uint32_t ta = tmem + 64u * (uint32_t)as, td = tmem + 256u + 64u * (uint32_t)ds;
#pragma unroll
          for (int gi = 0; gi < 8; ++gi)
            tc_mma_i8_ts(td + (uint32_t)TV_MMA_N * gi, ta + 8u * gi, tv_bdesc(bb + (uint32_t)gi * bst, 48u), idesc);
          tc_commit(&mdone[as]);
          KQ_TRACE_AT(k, 5);
        }
      }
      tc_commit(&mma_done);
      tv_drain_wait(&mma_done, 0, P.err);   // every MMA issued here has completed
    }
    __syncwarp();
  } else {
    // ---------------- warps 0-11: the prologue (activation digits -> B tiles), then their roles
    constexpr int NP = (TV_DQ_WARPS + TV_RO_WARPS) * 32;
    pdl_wait();
    tv_prologue<NP>(P, sm, L, s_redd, threadIdx.x);
    fence_proxy_async();   // the B tiles are read by the tensor cores
    named_bar(1, NP);
    if (threadIdx.x == 0) {
      mbar_arrive(&b_ready);
      KQ_TRACE_AT(255, 0);
    }
  if (warp < TV_DQ_WARPS) {
    // ---------------- A-digit writers: thread (row r of the warp's TMEM lane quarter, half hh of
    // the super-block); the thread of half 0 also copies its row's header for the read-back
    const int qd = warp & 3, hh = warp >> 2, r = 32 * qd + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * qd) << 16);
    for (int k = 0; k < n; ++k) {
      const int slot = k % TV_RS, as = k % TV_AS, hs = k % TV_HS;
      if (!__all_sync(0xffffffffu, tv_wait(&raw_full[slot], (uint32_t)(k / TV_RS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f, 64)))
        break;
      // A slot free (the MMAs of unit k - TV_AS have completed) and D slot free (the read-back of
      // unit k - TV_AS has its D and header; it reads the header slot (k - TV_AS) % TV_HS, and the
      // header slot k % TV_HS was last read by the read-back of unit k - TV_HS, earlier still)
      if (k >= TV_AS &&
          !(__all_sync(0xffffffffu, tv_wait(&mdone[as], (uint32_t)((k / TV_AS) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f, 64)) &&
            __all_sync(0xffffffffu, tv_wait(&d_free[as], (uint32_t)((k / TV_AS) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f, 64))))
        break;
      tc_fence_after();
      if (threadIdx.x == 0) KQ_TRACE_AT(k, 0);
      const long long u = u0 + k;
      const bool q4 = P.seg[seg_of((int)(u / G))].w.type == Q4K;
      const uint8_t* st = raw_ring + (size_t)slot * TV_RAW_BYTES;
      const uint32_t ta = tl + 64u * (uint32_t)as + 32u * (uint32_t)hh;
      if (q4) {
        if (hh == 0) hdr[hs * TV_ROWS + r] = lds128(st + TV_ST_HDR + 16 * r);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          // the 32 bytes of (hh, c): low nibbles = sub-block 4hh + 2c, high = 4hh + 2c + 1
          const uint8_t* b = st + c * TV_ST_C1;
          const uint4 W0 = lds128(b + tv_sw64(r, 2 * hh)), W1 = lds128(b + tv_sw64(r, 2 * hh + 1));
          const uint32_t wd[8] = {W0.x, W0.y, W0.z, W0.w, W1.x, W1.y, W1.z, W1.w};
          uint32_t lo[8], hi[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) { lo[i] = wd[i] & 0x0F0F0F0Fu; hi[i] = wd[i] & 0xF0F0F0F0u; }
          tc_st8(ta + 16u * c, lo);
          tc_st8(ta + 16u * c + 8u, hi);
        }
      } else {
        if (hh == 0) {
          hdr[hs * TV_ROWS + r] = lds128(st + TV_ST_SC + 16 * r);
          hdrd[hs * TV_ROWS + r] = *reinterpret_cast<const uint16_t*>(st + TV_ST_D + 2 * r);
        }
        const uint4 H0 = lds128(st + TV_ST_QH + tv_sw64(r, 2 * hh)), H1 = lds128(st + TV_ST_QH + tv_sw64(r, 2 * hh + 1));
        const uint32_t qh[8] = {H0.x, H0.y, H0.z, H0.w, H1.x, H1.y, H1.z, H1.w};
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          const uint8_t* lq = st + m * TV_ST_C1;
          const uint4 L0 = lds128(lq + tv_sw64(r, 2 * hh)), L1 = lds128(lq + tv_sw64(r, 2 * hh + 1));
          const uint32_t ql[8] = {L0.x, L0.y, L0.z, L0.w, L1.x, L1.y, L1.z, L1.w};
#pragma unroll
          for (int nib = 0; nib < 2; ++nib) {
            // group k = 2 nib + m: ql chunk m, nibble nib, qh bits 2k
            const int kk = 2 * nib + m;
            uint32_t q6[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              q6[i] = ((ql[i] >> (4 * nib)) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * kk)) & 0x03030303u) << 4);
            tc_st8(ta + 8u * kk, q6);
          }
        }
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[as]);
        mbar_arrive(&raw_empty[slot]);
        if (k < 50) KQ_TRACE_AT(100 + k, warp);
      }
      if (threadIdx.x == 0) KQ_TRACE_AT(k, 1);
    }
  } else {
    // ---------------- read-back warps (thread = row r of the warp's TMEM lane quarter): prologue,
    // then per unit the row's int32 dot products with the scales applied, tile flushes, epilogues
    const int tid = threadIdx.x - TV_DQ_WARPS * 32, qd = warp & 3, r = 32 * qd + lane;
    constexpr int NT = TV_RO_WARPS * 32;
    const uint32_t tl = tmem + ((uint32_t)(32 * qd) << 16);
    const float* s3a = reinterpret_cast<const float*>(sm + L.s3);
    const float* x32 = reinterpret_cast<const float*>(sm + L.x32);
    const int4* c16 = reinterpret_cast<const int4*>(sm + L.c16);
    const int tf0 = (int)(u0 / G);   // this CTA's first tile
    float acc = 0.f;
    bool ok = true;
    // Header slot k % TV_HS is rewritten (unit k + TV_HS) only after the writers of unit k + TV_HS
    // saw the D release of unit k + TV_HS - TV_DS, which follows this read-back's release: the
    // header is read before that release.
    auto readout = [&](int k) -> bool {
      const int ds = k % TV_DS, hs = k % TV_HS;
      if (!__all_sync(0xffffffffu, tv_wait(&h_full[hs], (uint32_t)(k / TV_HS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f, 32)))
        return false;
      const uint4 H = hdr[hs * TV_ROWS + r];
      const uint32_t Hd = hdrd[hs * TV_ROWS + r];
      if (!__all_sync(0xffffffffu, tv_wait(&mdone[ds], (uint32_t)(k / TV_DS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f, 32)))
        return false;
      tc_fence_after();
      if (tid == 0) KQ_TRACE_AT(k, 2);
      const long long u = u0 + k;
      const int g = (int)(u % G);
      const bool q4 = P.seg[seg_of((int)(u / G))].w.type == Q4K;
      const uint32_t td = tl + 256u + 64u * (uint32_t)ds;
      int D0[32], D1[32];   // groups 0-3 and 4-7, 8 columns each
      tc_ld32_nw(td, D0);
      tc_ld32_nw(td + 32u, D1);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_free[ds]);
      const float s3 = s3a[g];
      int P3[3] = {0, 0, 0};
      if (q4) {
        const float d = h2f_bits(H.x & 0xFFFFu), dmin = h2f_bits(H.x >> 16);
        const uint32_t sc0 = H.y & 0x3F3F3F3Fu, sc1 = (H.w & 0x0F0F0F0Fu) | ((H.y >> 2) & 0x30303030u);
        const uint32_t mn0 = H.z & 0x3F3F3F3Fu, mn1 = ((H.w >> 4) & 0x0F0F0F0Fu) | ((H.z >> 2) & 0x30303030u);
        float Qm = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {   // sub-block j: high nibble if j odd (entered as 16 q)
          const int* Dj = j < 4 ? &D0[8 * j] : &D1[8 * (j - 4)];
          const int c = tv_ubyte(j < 4 ? sc0 : sc1, j & 3) << ((j & 1) ? 0 : 4);
          P3[0] += c * Dj[0];
          P3[1] += c * Dj[1];
          P3[2] += c * Dj[2];
          Qm = __fmaf_rn((float)tv_ubyte(j < 4 ? mn0 : mn1, j & 3), x32[g * 8 + j], Qm);
        }
        const float Pf = planes_combine(P3);
        acc = __fadd_rn(acc, __fsub_rn(__fmul_rn(__fmul_rn(s3, 0.0625f), __fmul_rn(d, Pf)), __fmul_rn(s3, __fmul_rn(dmin, Qm))));
      } else {
        const float d = h2f_bits(Hd);
        const uint32_t sw[4] = {H.x, H.y, H.z, H.w};   // scale words [u = 2h + jh][k]
#pragma unroll
        for (int gi = 0; gi < 8; ++gi) {   // group (h, k) = (gi >> 2, gi & 3)
          const int* Dj = gi < 4 ? &D0[8 * gi] : &D1[8 * (gi - 4)];
          const int h = gi >> 2, kk = gi & 3;
          const int sa = sbyte(sw[2 * h], kk), sb = sbyte(sw[2 * h + 1], kk);
          const int4 ca = c16[g * 16 + 2 * gi], cb = c16[g * 16 + 2 * gi + 1];
          P3[0] += sa * (Dj[0] - ca.x) + sb * (Dj[3] - cb.x);
          P3[1] += sa * (Dj[1] - ca.y) + sb * (Dj[4] - cb.y);
          P3[2] += sa * (Dj[2] - ca.z) + sb * (Dj[5] - cb.z);
        }
        acc = __fadd_rn(acc, __fmul_rn(s3, __fmul_rn(d, planes_combine(P3))));
      }
      if (tid == 0) KQ_TRACE_AT(k, 3);
      return true;
    };
    // end of tile t's units in this CTA: the epilogue if the CTA covered the whole tile, else the
    // partial and, for the last contributor, the merge in CTA order. Every read-back thread takes
    // the same barriers, also after a failure.
    auto flush = [&](int t, bool whole) {
      const bool good = named_bar_and(4, NT, ok && !*abort_f);
      const TvSeg& S = P.seg[seg_of(t)];
      const int row = (t - S.tile0) * TV_ROWS + r;
      float v = acc;
      bool fin = good && whole;
      if (good && !whole) {
        __stcg(P.part + ((size_t)cta * 2 + (t == tf0 ? 0 : 1)) * TV_ROWS + r, v);
        __threadfence();
        named_bar(3, NT);
        const int cf = tv_cta_of((long long)t * G, nct, U), cl = tv_cta_of((long long)t * G + G - 1, nct, U);
        if (tid == 0) s_last = atomicAdd(&P.ticket[t], 1) == cl - cf;
        named_bar(3, NT);
        fin = s_last;
        if (fin) {
          __threadfence();
          v = 0.f;
          for (int c = cf; c <= cl; ++c) {
            const int tfc = (int)(tv_unit0(c, nct, U) / G);
            v = __fadd_rn(v, __ldcg(P.part + ((size_t)c * 2 + (t == tfc ? 0 : 1)) * TV_ROWS + r));
          }
          if (tid == 0) P.ticket[t] = 0;
        }
      }
      if (fin) {
        const float vo = __shfl_xor_sync(0xffffffffu, v, 1);
        if (row < S.w.R) tv_epilogue(P, S, row, v, vo);
      }
      named_bar(4, NT);   // s_last is reused by the next flush
      acc = 0.f;
    };
    for (int k = 0; k < n; ++k) {
      if (ok) ok = readout(k);
      const long long u = u0 + k;
      const int t = (int)(u / G);
      if (k == n - 1 || (int)((u + 1) / G) != t) flush(t, u0 <= (long long)t * G && (int)(u % G) == G - 1);
    }
    if (tid == 0) KQ_TRACE_AT(255, 1);
  }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) KQ_TRACE_AT(0, 11);
  if (warp == TV_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, TV_TMEM_COLS);
  }
}

}  // namespace kq
