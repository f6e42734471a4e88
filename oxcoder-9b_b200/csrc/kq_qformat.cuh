// kq_qformat.cuh -- device layout of Q4_K / Q6_K matrices, the seeded synthetic generator, the
// GGUF -> device repack and the bit-exact dequantiser.
//
// Device layout ("kq layout"). A matrix of R rows (a multiple of 8) and C = 256*G columns is
// stored as R/8 tiles of 8 rows; a tile holds its rows' planes one after another, so a run of
// whole tiles is ONE contiguous range (one bulk copy per pipeline stage). Inside a tile:
//   p0  [8][2][G][4][16]   nibble bytes (Q4_K qs / Q6_K ql): chunk (c, g, u) holds GGUF block
//                          bytes 64h + 32c + 16jh + (0..15) of the nibble area, u = 2h + jh
//   p1  Q4_K: [8][G][16]   block header verbatim (d, dmin, 12 packed 6-bit scales/mins)
//       Q6_K: [8][G][64]   qh bytes verbatim (unit u's 16 bytes at 16u)
//   p2  Q6_K: [8][G][4][4] int8 scales, unit-major: [u][k] = GGUF scale 8h + 2k + jh
//   p3  Q6_K: [8][G]       fp16 d
// Thread "unit" u of block g covers the 64 columns 256g + 128h + 32k + 16jh + j', k = 0..3,
// j' = 0..15, for BOTH types, so one set of activation digits serves mixed-type launches.
// The byte count equals the GGUF byte count (144 or 210 per block); nothing is re-quantised.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include "kq_common.cuh"

namespace kq {

constexpr int Q4K = 12, Q6K = 14;

struct QView {
  const uint8_t* base;   // R/8 tiles
  int type, R, C, G;
  const uint8_t* tv;     // the unit-major copy of the tensor-core GEMV (kq_tmv.cuh), or null
};

__host__ __device__ inline int block_bytes(int type) { return type == Q4K ? 144 : 210; }
__host__ __device__ inline size_t plane_row_bytes(int type, int plane, int G) {
  if (plane == 0) return (size_t)128 * G;
  if (plane == 1) return (size_t)(type == Q4K ? 16 : 64) * G;
  if (plane == 2) return type == Q4K ? 0 : (size_t)16 * G;
  return type == Q4K ? 0 : (size_t)2 * G;
}
__host__ __device__ inline size_t tile_bytes(int type, int G) { return (size_t)8 * block_bytes(type) * G; }
// offset of plane p inside a tile
__host__ __device__ inline size_t tile_plane_off(int type, int G, int plane) {
  size_t o = 0;
  for (int p = 0; p < plane; ++p) o += 8 * plane_row_bytes(type, p, G);
  return o;
}
// Tiles are laid out so that the 8 rows of a tile can be read in parallel without shared-memory
// bank conflicts (the tensor-core GEMV reads the same columns of 8 or 16 rows at once), while one
// row stays conflict-free too (k_gemv reads consecutive chunks of one row). Every access is of
// whole 16-byte chunks or less, and a chunk moves only inside its 128-byte group (XOR with the
// row's index in its tile):
//   plane 0, both types (the nibbles, 128 G bytes a row): chunk q of row r8 at q ^ r8;
//   plane 1, Q4_K (16-byte block headers) and plane 2, Q6_K (16 int8 scales a block): chunk g of
//            row r8 at g ^ r8 when G is a multiple of 8 (rows then start on 128-byte boundaries);
//   plane 1, Q6_K (qh, 64 bytes a block): chunk q at q ^ r8 when G is even.
__host__ __device__ inline size_t p0_swz(int row, size_t off) { return off ^ ((size_t)(row & 7) << 4); }
__host__ __device__ inline size_t q4_p1_swz(int G, int row, size_t off) {
  return (G & 7) ? off : off ^ ((size_t)(row & 7) << 4);
}
__host__ __device__ inline size_t q6_qh_swz(int G, int row, size_t off) {
  return (G & 1) ? off : off ^ ((size_t)(row & 7) << 4);
}

// byte `off` of plane p of row `row` (offsets as in the unswizzled [8 rows][bytes] order of the
// plane), relative to a tile-aligned base holding row 0 of a tile
__host__ __device__ inline size_t row_plane_off(int type, int G, int row, int plane, size_t off) {
  const size_t t = (size_t)(row >> 3) * tile_bytes(type, G) + tile_plane_off(type, G, plane) +
                   (size_t)(row & 7) * plane_row_bytes(type, plane, G);
  if (plane == 0) return t + p0_swz(row, off);
  if (type == Q4K && plane == 1) return t + q4_p1_swz(G, row, off);
  if (type == Q6K && plane == 1) return t + q6_qh_swz(G, row, off);
  if (type == Q6K && plane == 2) return t + q4_p1_swz(G, row, off);
  return t + off;
}

// ------------------------------------------------------------------------------------------
// Seeded generator. Specification (shared with the CPU oracle's own implementation): draw i of
// stream s under seed S is fin(base(S, s) + (i + 1) * GAMMA), fin = splitmix64's output mix.
// Values use exact integer work or single IEEE fp32 operations, so host and device agree.
constexpr uint64_t KQ_GAMMA = 0x9E3779B97F4A7C15ull;
__host__ __device__ inline uint64_t gen_fin(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t gen_base(uint64_t seed, uint64_t stream) {
  return gen_fin(gen_fin(seed * KQ_GAMMA + 0x632BE59BD9B4E019ull) ^ (stream * 0xD1B54A32D192ED03ull));
}
__host__ __device__ inline uint64_t gen_draw(uint64_t base, uint64_t i) { return gen_fin(base + (i + 1) * KQ_GAMMA); }

__device__ inline float gen_unif24(uint32_t u24, float lo, float span) {
  const float u = (float)u24 * 0x1p-24f;
  return __fadd_rn(lo, __fmul_rn(u, span));
}
__device__ inline float gen_nrm(uint64_t base, uint64_t i) {
  long long s = 0;
  for (int k = 0; k < 6; k++) {
    const uint64_t r = gen_draw(base, i * 6 + (uint64_t)k);
    s += (long long)(r & 0xFFFFFF) + (long long)((r >> 24) & 0xFFFFFF);
  }
  return (float)(s - 6ll * 16777216ll) * 0x1p-24f;
}
__device__ inline uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Q4_K block bi of a stream (19 draws), GGUF byte order.
__device__ inline void gen_q4k_block(uint64_t base, uint64_t bi, uint8_t* b) {
  const uint64_t k0 = bi * 19;
  const uint64_t r0 = gen_draw(base, k0), r1 = gen_draw(base, k0 + 1), r2 = gen_draw(base, k0 + 2);
  const uint16_t d = f2h_bits(gen_unif24((uint32_t)(r0 & 0xFFFFFF), 1e-4f, 3e-4f));
  const uint16_t dm = f2h_bits(gen_unif24((uint32_t)((r0 >> 24) & 0xFFFFFF), 1e-4f, 3e-4f));
  b[0] = (uint8_t)d; b[1] = (uint8_t)(d >> 8); b[2] = (uint8_t)dm; b[3] = (uint8_t)(dm >> 8);
  int sc[8], mn[8];
  for (int k = 0; k < 8; k++) { sc[k] = (int)((r1 >> (8 * k)) & 63); mn[k] = (int)((r2 >> (8 * k)) & 63); }
  uint8_t* s = b + 4;
  for (int k = 0; k < 4; k++) {
    s[k] = (uint8_t)(sc[k] | ((sc[k + 4] >> 4) << 6));
    s[k + 4] = (uint8_t)(mn[k] | ((mn[k + 4] >> 4) << 6));
    s[k + 8] = (uint8_t)((sc[k + 4] & 15) | ((mn[k + 4] & 15) << 4));
  }
  for (int w = 0; w < 16; w++) {
    const uint64_t r = gen_draw(base, k0 + 3 + (uint64_t)w);
    for (int i = 0; i < 8; i++) b[16 + 8 * w + i] = (uint8_t)(r >> (8 * i));
  }
}
// Q6_K block bi (27 draws), GGUF byte order.
__device__ inline void gen_q6k_block(uint64_t base, uint64_t bi, uint8_t* b) {
  const uint64_t k0 = bi * 27;
  for (int w = 0; w < 24; w++) {
    const uint64_t r = gen_draw(base, k0 + (uint64_t)w);
    for (int i = 0; i < 8; i++) b[8 * w + i] = (uint8_t)(r >> (8 * i));
  }
  const uint64_t s0 = gen_draw(base, k0 + 24), s1 = gen_draw(base, k0 + 25), rd = gen_draw(base, k0 + 26);
  for (int i = 0; i < 16; i++) {
    const uint64_t r = i < 8 ? s0 : s1;
    b[192 + i] = (uint8_t)(int8_t)((int)((r >> (8 * (i & 7))) & 127) - 64);
  }
  const uint16_t d = f2h_bits(gen_unif24((uint32_t)(rd & 0xFFFFFF), 1e-4f, 3e-4f));
  b[208] = (uint8_t)d; b[209] = (uint8_t)(d >> 8);
}

// ------------------------------------------------------------------------------------------
// Row maps: device row of source row `s` of the tensor being written.
//   RM_IDENT      dev = s
//   RM_ROPE_PAIR  rows (i, i + hd/2) of each head become adjacent (2i, 2i + 1), so the fused
//                 epilogue of the projection can rotate a pair in one thread
//   RM_INTERLEAVE dev = 2s + which (gate rows even, up rows odd: SwiGLU pairs)
enum { RM_IDENT = 0, RM_ROPE_PAIR = 1, RM_INTERLEAVE = 2 };
__host__ __device__ inline int map_row(int s, int mode, int arg) {
  if (mode == RM_ROPE_PAIR) {
    const int hd = arg, hh = s / hd, e = s % hd, half = hd / 2;
    return hh * hd + 2 * (e % half) + e / half;
  }
  if (mode == RM_INTERLEAVE) return 2 * s + arg;
  return s;
}

struct QViewW {   // writable view
  uint8_t* base;
  int type, R, C, G;
};

// Scatter GGUF block b of device row d, block g into the planes.
__device__ inline void scatter_block(const QViewW& m, int d, int g, const uint8_t* b) {
  const int G = m.G, t = m.type;
  if (t == Q4K) {
    uint8_t* meta = m.base + row_plane_off(t, G, d, 1, (size_t)g * 16);   // 16 contiguous bytes
    for (int i = 0; i < 16; i++) meta[i] = b[i];
    for (int o = 0; o < 128; o++) {
      const int h = o >> 6, c = (o >> 5) & 1, jh = (o >> 4) & 1, jp = o & 15;
      m.base[row_plane_off(t, G, d, 0, (size_t)c * 64 * G + (size_t)g * 64 + (2 * h + jh) * 16 + jp)] = b[16 + o];
    }
  } else {
    for (int o = 0; o < 128; o++) {
      const int h = o >> 6, c = (o >> 5) & 1, jh = (o >> 4) & 1, jp = o & 15;
      m.base[row_plane_off(t, G, d, 0, (size_t)c * 64 * G + (size_t)g * 64 + (2 * h + jh) * 16 + jp)] = b[o];
    }
    for (int o = 0; o < 64; o++) m.base[row_plane_off(t, G, d, 1, (size_t)g * 64 + o)] = b[128 + o];
    uint8_t* sc = m.base + row_plane_off(t, G, d, 2, (size_t)g * 16);   // 16 contiguous bytes
    for (int h = 0; h < 2; h++)
      for (int jh = 0; jh < 2; jh++)
        for (int k = 0; k < 4; k++) sc[(2 * h + jh) * 4 + k] = b[192 + 8 * h + 2 * k + jh];
    uint8_t* dd = m.base + row_plane_off(t, G, d, 3, (size_t)g * 2);
    dd[0] = b[208]; dd[1] = b[209];
  }
}

// One thread per (source row, block): block from `src` (GGUF row-major bytes of R_src rows) or,
// if src == nullptr, from the generator (stream, seed); written to device row map_row(s).
// A tensor-parallel shard draws the blocks of the full matrix it is a slice of: generator block
// index (s + sh.row_off) * sh.G_src + (g + sh.g_off), with G_src the full matrix's super-blocks.
struct ShardMap {
  int row_off, g_off, G_src;   // {0, 0, G}: the whole matrix
  int pack;                    // 1: `src` is in the Kindi pack's 8-row interleave (q4kernels.h:8-10),
                               // block (row, g) at ((row / 8) * G + g) * 8 + row % 8
};
__global__ void k_qmat_write(QViewW m, int R_src, const uint8_t* __restrict__ src, uint64_t base,
                             int mode, int arg, ShardMap sh) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)R_src * m.G) return;
  const int s = (int)(idx / m.G), g = (int)(idx % m.G);
  uint8_t b[210];
  const int bs = block_bytes(m.type);
  if (src) {
    const size_t blk = sh.pack ? ((size_t)(s >> 3) * m.G + g) * 8 + (s & 7) : (size_t)s * m.G + g;
    const uint8_t* p = src + blk * bs;
    for (int i = 0; i < bs; i++) b[i] = p[i];
  } else if (m.type == Q4K) {
    gen_q4k_block(base, (uint64_t)(s + sh.row_off) * sh.G_src + (uint64_t)(g + sh.g_off), b);
  } else {
    gen_q6k_block(base, (uint64_t)(s + sh.row_off) * sh.G_src + (uint64_t)(g + sh.g_off), b);
  }
  scatter_block(m, map_row(s, mode, arg), g, b);
}

// fp32 vector mu + sigma * z, z ~ approx N(0,1) (Irwin-Hall 12), two roundings.
__global__ void k_gen_normal(float* y, long long n, float mu, float sigma, uint64_t base) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __fadd_rn(mu, __fmul_rn(sigma, gen_nrm(base, (uint64_t)i)));
}
// fp16 ~ N(0,1) values, written at dst[i] for i in [0, n).
__global__ void k_gen_half_normal(__half* y, long long n, uint64_t base) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2half_rn(gen_nrm(base, (uint64_t)i));
}

// ------------------------------------------------------------------------------------------
// Exact dequantisation of one element (row, col) from the device layout, in the reference's
// operation order (q4kernels.h:12-33): Q4_K w = fl(fl(d*sc)*q) - fl(dmin*mn); Q6_K
// w = fl(d*scale)*(q-32).
__device__ inline float dequant_elem(const QView& m, int row, int col) {
  const int G = m.G, t = m.type, g = col >> 8, e = col & 255;
  const int h = e >> 7, k6 = (e >> 5) & 3, j = e & 31, jh = j >> 4, jp = j & 15, u = 2 * h + jh;
  if (t == Q4K) {
    const uint8_t* meta = m.base + row_plane_off(t, G, row, 1, (size_t)g * 16);
    const float d = h2f_bits(meta[0] | (meta[1] << 8)), dm = h2f_bits(meta[2] | (meta[3] << 8));
    const uint8_t* s = meta + 4;
    const int k = 4 * h + k6;
    const int sc = k < 4 ? (s[k] & 63) : ((s[k + 4] & 15) | ((s[k - 4] >> 6) << 4));
    const int mn = k < 4 ? (s[k + 4] & 63) : ((s[k + 4] >> 4) | ((s[k] >> 6) << 4));
    const uint8_t byte = m.base[row_plane_off(t, G, row, 0, (size_t)(k6 >> 1) * 64 * G + (size_t)g * 64 + u * 16 + jp)];
    const int q = (byte >> ((k6 & 1) * 4)) & 15;
    const float ds = __fmul_rn(d, (float)sc), ms = __fmul_rn(dm, (float)mn);
    return __fsub_rn(__fmul_rn(ds, (float)q), ms);
  }
  const uint8_t lob = m.base[row_plane_off(t, G, row, 0, (size_t)(k6 & 1) * 64 * G + (size_t)g * 64 + u * 16 + jp)];
  const int low = (lob >> ((k6 >> 1) * 4)) & 15;
  const int high = (m.base[row_plane_off(t, G, row, 1, (size_t)g * 64 + u * 16 + jp)] >> (2 * k6)) & 3;
  const int scale = (int8_t)m.base[row_plane_off(t, G, row, 2, (size_t)g * 16 + u * 4 + k6)];
  const uint8_t* dp = m.base + row_plane_off(t, G, row, 3, (size_t)g * 2);
  const float d = h2f_bits(dp[0] | (dp[1] << 8));
  return __fmul_rn(__fmul_rn(d, (float)scale), (float)((low | (high << 4)) - 32));
}

__global__ void k_qmat_dequant(QView m, int row0, int nrows, float* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)nrows * m.C) return;
  const int r = (int)(i / m.C), c = (int)(i % m.C);
  out[i] = dequant_elem(m, row0 + r, c);
}

}  // namespace kq
