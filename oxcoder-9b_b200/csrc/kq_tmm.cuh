// kq_tmm.cuh -- fused-dequant GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulators)
// for the multi-token passes: Y[M][R] = X[M][C] W^T with W in the kq Q4_K / Q6_K device layout and
// M <= 128 tokens (the verification pass over a draft tree, the M-row matrix product).
//
// Precision. The Kindi CPU path dequantises every weight in fp32 (w = (d*sc)*q - dmin*mn, or
// (d*scale)*(q6 - 32); q4kernels.h:19-30) and accumulates in fp32. Here each weight w and each
// activation x is carried as two fp16 numbers, hi = fp16(v) and lo = fp16(v - hi) (about 22
// significant bits), and every 16-column K step issues two MMAs: hi(w) * [hi(x); lo(x)] (the
// activation stage stacks the hi and the lo token rows, so one MMA of N = 2 Npad forms both
// products) and lo(w) * hi(x), each product in its own fp32 TMEM accumulator (the small
// corrections are not rounded against the large partial sums) and summed in the epilogue. The
// dropped lo*lo term is below 2^-22 of the product, so the result is within a few fp32 roundings
// of the fp32 dot product. The weights' hi/lo pairs live in tensor memory (the MMA's A operand),
// written by the dequantising warps with tcgen05.st; only the raw bytes and the activations pass
// through shared memory. That is the split-weight form; Q4_K row tiles of inputs that come with
// sub-block sums take the exact form instead (A = q * sc, exact in fp16, one MMA per K step; d
// and the minimum term applied in fp32 outside the tensor core; see TM_XAS below).
//
// CTA = 128 weight rows (16 tiles of the kq layout) x all tokens x a contiguous range of super-
// blocks (split-K over CTAs; the last CTA of a row tile sums the fp32 partials in split order, so
// the result does not depend on which CTA finishes last). Warp roles (352 threads):
//   warps 0-7  dequantise: raw super-block bytes (shared memory) -> hi/lo fp16 A sub-stages of
//              64 columns in tensor memory (thread = weight row); then the epilogue
//   warp 8     raw loader: cp.async of each super-block's bytes for the 128 rows into a padded ring
//              (row strides 144 B / 208 B = an odd number of 16-byte units: conflict-free reads)
//   warp 9     TMEM allocation; lane 0 issues tcgen05.mma (split form: 2 x 8 per 128-column
//              sub-stage; exact form: 16 per super-block) and commits each stage's completion to
//              the barriers that free its A and X buffers (exact form: and its accumulator buffer)
//   warp 10    activation loader: one cp.async.bulk per 128-column sub-stage of the packed X (exact
//              form: per super-block, plus its sub-block sums), into its own ring (as deep as
//              shared memory allows), freed by the MMA commits
// Every wait is bounded; on a timeout the CTA records the error, stops issuing work, drains what
// it issued and frees its tensor memory before it exits.
#pragma once
#include "kq_common.cuh"
#include "kq_qformat.cuh"
#include "kq_gemv.cuh"

namespace kq {

// ------------------------------------------------------------------------------ packed activations
// The B operand of the GEMM: for every 64-column group, an hi plane then a lo plane, each Npad
// token rows of 128 bytes (64 fp16) in the SWIZZLE_128B K-major layout: the 16-byte chunk j of
// token t's row sits at chunk position j ^ (t & 7). Npad is a multiple of 16 (the MMA's N).
__host__ __device__ inline size_t xp_group_halves(int Npad) { return (size_t)2 * 64 * Npad; }
__host__ __device__ inline size_t xp_halves(int Npad, int C) { return (size_t)(C / 64) * xp_group_halves(Npad); }
__device__ __forceinline__ size_t xp_off(int Npad, int tok, int col) {
  const int q = col >> 6, j8 = (col >> 3) & 7;
  return (size_t)q * xp_group_halves(Npad) + (size_t)tok * 64 + (size_t)(((j8 ^ (tok & 7)) << 3) | (col & 7));
}
__device__ __forceinline__ void xp_store(__half* xp, int Npad, int tok, int col, float v) {
  const __half hi = __float2half_rn(v);
  const __half lo = __float2half_rn(__fsub_rn(v, __half2float(hi)));
  const size_t o = xp_off(Npad, tok, col);
  xp[o] = hi;
  xp[o + (size_t)64 * Npad] = lo;
}
// Sub-block sums of the packed rows, for the exact form of the GEMM: xsum[g][t][b] = the fp32 sum
// of token t's packed values over columns 256 g + 32 b .. + 31. The caller holds the 8 packed
// values of chunk c (columns 8c .. 8c + 7) of token t; the four chunks of a sub-block sit in four
// adjacent lanes, and every lane of the warp takes part.
__device__ __forceinline__ void xp_sub_sum(float* xsum, int Npad, int t, int c, const float (&x)[8]) {
  float s = __fadd_rn(__fadd_rn(__fadd_rn(x[0], x[1]), __fadd_rn(x[2], x[3])),
                      __fadd_rn(__fadd_rn(x[4], x[5]), __fadd_rn(x[6], x[7])));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
  if ((c & 3) == 0) {
    const int sb = c >> 2;
    xsum[((size_t)(sb >> 3) * Npad + t) * 8 + (sb & 7)] = s;
  }
}

// Per-token range scaling of the packed activations. hi = fp16(x) overflows for |x| > 65504 (hi +
// lo then turns into inf - inf in the MMA), and below 2^-14 hi and lo lose bits to fp16's
// subnormal range. A producer (the SwiGLU output, a caller's fp32 rows, a norm output) packs token
// t's row scaled by 2^-e_t, e_t = floor(log2 of the row's largest magnitude, or a bound of it) - 14,
// so that magnitude lands in [2^14, 2^15), and records 2^e_t; the GEMM epilogue multiplies token
// t's results by it. Powers of two are exact. e_t is kept >= -100 (2^100 and 2^-100 are normal
// floats); a zero row, NaN and inf keep e_t = 0 (non-finite values propagate).
__device__ __forceinline__ int xp_scale_exp(float amax) {
  if (!(amax > 0.f) || amax > 3.0e38f) return 0;
  const int e = (int)((__float_as_uint(amax) >> 23) & 255u) - 127 - 14;   // floor(log2 amax) - 14
  return e < -100 ? -100 : e;
}
__device__ __forceinline__ float xp_pow2(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

// ------------------------------------------------------------------------------ tcgen05 wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (both operands fp16), fp32 accumulate.
__device__ __forceinline__ void tc_mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive once on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 8 consecutive fp32 columns of this thread's TMEM lane (the warp's 32-lane quarter), waited.
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r0, r1, r2, r3, r4, r5, r6, r7;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3), "=r"(r4), "=r"(r5), "=r"(r6), "=r"(r7)
      : "r"(taddr)
      : "memory");
  v[0] = __uint_as_float(r0); v[1] = __uint_as_float(r1); v[2] = __uint_as_float(r2); v[3] = __uint_as_float(r3);
  v[4] = __uint_as_float(r4); v[5] = __uint_as_float(r5); v[6] = __uint_as_float(r6); v[7] = __uint_as_float(r7);
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row atoms of 1024 bytes stacked along
// M/N (stride 1024), start address 16-byte granular (fields: start >> 4 at bit 0, leading offset
// at bit 16 (unused by swizzled K-major layouts), stride >> 4 at bit 32, descriptor version 1 at
// bit 46, layout type 2 = 128-byte swizzle at bit 61).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: fp32 D (bit 4), fp16 A and B (formats 0), both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t tc_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// cp.async of 16 (or 4) bytes, zero-filled when src_bytes = 0; L2 evict-first for streamed weights.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
// Arrive on `bar` (counted in its initial count) when this thread's earlier cp.asyncs complete.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Named barrier that also ANDs a predicate over the participating threads (uniform result).
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, %2, %3, q;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r) : "r"((uint32_t)v), "r"(id), "r"(nthreads) : "memory");
  return r != 0;
}

// ------------------------------------------------------------------------------ the GEMM
struct BatchParams {                   // per-token data of a pass
  int M;
  const int* slot;                     // [M] K/V slot
  const int* rpos;                     // [M] rotary position
  const unsigned long long* mask;      // [M][2] ancestor masks relative to tree_base
  int tree_base;
  const int* seq;                      // [M] sequence of each token (batched decode), or null: 0
};

constexpr int TM_ROWS = 128;                       // weight rows per CTA (the MMA's M)
constexpr int TM_DQ_WARPS = 8;                     // dequantising / epilogue warps
constexpr int TM_THREADS = (TM_DQ_WARPS + 3) * 32; // + raw loader, MMA, activation loader
constexpr int TM_RS = 4;                           // raw super-block stages in flight
constexpr int TM_AS = 3;                           // A sub-stages (128 columns each) in tensor memory, at most
constexpr int TM_XS_MAX = 8;                       // activation sub-stage buffers (fill the rest)
constexpr int TM_RAW_Q4 = 144, TM_RAW_Q6 = 208;    // raw row strides (odd multiples of 16 B)
constexpr int TM_RAW_BYTES = TM_ROWS * TM_RAW_Q6;  // one raw stage
constexpr int TM_MAXN = 128;                       // tokens per GEMM (Npad)
// A sub-stage is 128 K columns (half a super-block). Tensor memory (512 columns of 128 lanes x
// 32 bits): accumulators first, hi(w) * hi(x) in columns [0, Npad) and the corrections
// hi(w) * lo(x) + lo(w) * hi(x) in [Npad, 2 Npad) (the first MMA of a K step has N = 2 Npad: the
// activation stage holds the hi token rows then the lo rows); then A sub-stages of 128 columns
// from tmm_acol(Npad): 64 columns of hi fp16 pairs, 64 of lo, lane = weight row, column c = K
// elements 2c, 2c + 1. Npad <= 64: 3 A stages; Npad <= 128: 2.
constexpr uint32_t TM_TMEM_COLS = 512, TM_ASTAGE_COLS = 128;
__host__ __device__ constexpr uint32_t tmm_acol(int Npad) { return Npad <= 64 ? 128u : 256u; }
__host__ __device__ constexpr int tmm_as(int Npad) { return Npad <= 64 ? 3 : 2; }
static_assert(128 + 3 * TM_ASTAGE_COLS <= TM_TMEM_COLS && 256 + 2 * TM_ASTAGE_COLS <= TM_TMEM_COLS, "tensor memory plan");
// Exact-integer form (Q4_K row tiles, Npad <= 64, activations packed with their sub-block sums).
// A holds q * sc, an integer <= 945 and so exact in fp16: one MMA per K step (N = 2 Npad against
// the hi and the lo token rows) and a quarter of the dequantisation work. The super-block scale d
// and the minimum term are applied outside the tensor core: each super-block accumulates into one
// of two buffers of tensor memory (columns [0, 128) and [128, 256): A * hi(x) in the first Npad
// columns, A * lo(x) in the next), which the dequantising warps read back, scale by d and add to
// registers while the next super-block accumulates in the other buffer; the minimum term
// dmin * mn * (sum of x over the sub-block) is an fp32 product with the sub-block sums that the
// packer wrote. Then 2 A stages of one super-block (128 columns of q * sc fp16 pairs) from column
// 256. Every hand-off (A stage, activation stage, accumulator buffer) is per super-block: the
// waits and commits of the single MMA-issuing thread, not the MMAs, set the pace of this kernel.
constexpr int TM_XAS = 2, TM_SR = 4;               // A stages (super-blocks); sub-block-sum stages
constexpr uint32_t TM_XD_COLS = 128, TM_XA0 = 256, TM_XASTAGE_COLS = 128;
constexpr int TM_AS_MAX = TM_XAS > TM_AS ? TM_XAS : TM_AS;
static_assert(TM_XA0 + TM_XAS * TM_XASTAGE_COLS <= TM_TMEM_COLS && 2 * TM_XD_COLS <= TM_XA0, "tensor memory plan (exact form)");
static_assert(TM_RAW_BYTES % 1024 == 0, "rings must keep 1024-byte alignment");

struct TmmSeg {
  QView w;
  int epi;
  int tile0;           // first row tile (of TM_ROWS rows) of this segment in the grid
  float* out_f;        // F32 / ROPE_Q output
  __half* out_h;       // ROPE_K / V: this layer's cache [n_kv][ctx][hd]
};
struct TmmParams {
  TmmSeg seg[KQ_MAX_SEG];
  int nseg, ntiles;    // row tiles over all segments
  int C, G, nsplit;    // K = C columns, G super-blocks, split over nsplit CTAs
  int M, Npad;         // tokens, MMA N (multiple of 16)
  int xs;              // activation ring stages (1..TM_XS_MAX), see tmm_smem
  const __half* xp;    // packed activations (xp_off layout)
  const float* xscale; // per token: the power of two its packed row was divided by (null: none)
  const float* xsum;   // sub-block sums of the packed rows [G][Npad][8] (xp_sub_sum), or null
  BatchParams B;
  int out_ld;          // row length of the fp32 outputs
  const float* cos_t;
  const float* sin_t;
  int hd, ctx;
  int nkv;             // KV heads per sequence in the cache ([seq][nkv][ctx][hd]; one sequence: any)
  float* part;         // split-K partials [nsplit][Npad][ntiles * TM_ROWS]
  int* ticket;         // [ntiles], zero between launches
  int* err;
  int trace_id;        // launch index for the optional phase trace (KQ_TRACE builds)
};

// Dynamic shared memory: 1024-byte alignment slack, raw ring, `xs` activation stages of
// 512 * Npad bytes (two 64-column groups; 1024-byte aligned: SWIZZLE_128B atoms), Q6_K d words,
// TM_SR stages of one super-block's sub-block sums (32 * Npad bytes; exact form).
__host__ __device__ inline size_t tmm_smem_fixed() {
  return 1024 + (size_t)TM_RS * TM_RAW_BYTES + (size_t)TM_RS * TM_ROWS * 4;
}
__host__ __device__ inline size_t tmm_smem(int Npad, int xs) {
  return tmm_smem_fixed() + (size_t)xs * 512 * Npad + (size_t)TM_SR * 32 * Npad;
}
// The deepest activation ring that fits `budget` bytes of dynamic shared memory.
__host__ __device__ inline int tmm_xs(int Npad, size_t budget) {
  const size_t fixed = tmm_smem_fixed() + (size_t)TM_SR * 32 * Npad;
  const size_t room = budget > fixed ? budget - fixed : 0;
  const int xs = (int)(room / ((size_t)512 * Npad));
  return xs < 1 ? 0 : xs > TM_XS_MAX ? TM_XS_MAX : xs;
}

__device__ __forceinline__ uint64_t tm_clock_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after TM_WAIT_NS of wall time (or KQ_WAIT_LIMIT polls), or at once when
// another role of the CTA has flagged a failure. Every wait of the pipeline normally ends in
// microseconds.
constexpr uint64_t TM_WAIT_NS = 2000000000ull;
__device__ __forceinline__ bool tm_wait(uint64_t* bar, uint32_t parity, int* err, int bit, volatile int* abort_f) {
  uint64_t t0 = 0;
  for (uint32_t it = 0; it < KQ_WAIT_LIMIT; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255) == 255) {
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

// The same bound with non-suspending probes (mbarrier.test_wait), for the single MMA-issuing
// thread, whose waits are usually already satisfied: measured ~5 % faster per super-block than
// try_wait in the exact form.
__device__ __forceinline__ bool tm_spin(uint64_t* bar, uint32_t parity, int* err, int bit, volatile int* abort_f) {
  uint64_t t0 = 0;
  for (uint32_t it = 0; it < KQ_WAIT_LIMIT; ++it) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((it & 255) == 255) {
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
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, fp32 accumulate (A read from tensor memory).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// 16 consecutive 32-bit columns of this thread's TMEM lane (the warp's 32-lane quarter).
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// Byte e of x (a value < 2^8) as the float 2^23 + value (exact).
__device__ __forceinline__ float tm_magic(uint32_t x, int e) {
  return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540u | (uint32_t)e));
}
__device__ __forceinline__ void tm_split(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  hi = h2u(h);
  lo = h2u(__floats2half2_rn(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y)));
}
// fp32 rows x [M][ld] (C columns) -> packed activations, one CTA per token, each row scaled as
// xp_scale_exp says; scale[t] = 2^e_t. Tokens M..Npad-1 are left as they are (their GEMM columns
// are never stored).
constexpr int XP_THREADS = 256;
struct XPackParams {
  const float* x;      // [M][ld] rows, C columns (C and ld multiples of 8)
  int ld, C, Npad;
  __half* xp;          // packed activations
  float* scale;        // [M]
  float* xsum;         // sub-block sums (xp_sub_sum; C a multiple of 256), or null
};
__global__ void __launch_bounds__(XP_THREADS) k_xpack_tok(const __grid_constant__ XPackParams P) {
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float red[XP_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const float4* row = reinterpret_cast<const float4*>(P.x + (size_t)t * P.ld);
  const int nch = P.C / 8, Npad = P.Npad;
  __half* xp = P.xp;
  float mx = 0.f;
  for (int c = tid; c < nch; c += XP_THREADS) {
    const float4 a = row[2 * c], b = row[2 * c + 1];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < XP_THREADS / 32; ++w) mx = fmaxf(mx, red[w]);
  const int e = xp_scale_exp(mx);
  const float inv = xp_pow2(-e);
  for (int c = tid; c < nch; c += XP_THREADS) {   // with sums: nch is a multiple of 32 (whole warps)
    const float4 a = row[2 * c], b = row[2 * c + 1];
    const float x[8] = {__fmul_rn(a.x, inv), __fmul_rn(a.y, inv), __fmul_rn(a.z, inv), __fmul_rn(a.w, inv),
                        __fmul_rn(b.x, inv), __fmul_rn(b.y, inv), __fmul_rn(b.z, inv), __fmul_rn(b.w, inv)};
    uint4 hi, lo;
    tm_split(x[0], x[1], hi.x, lo.x);
    tm_split(x[2], x[3], hi.y, lo.y);
    tm_split(x[4], x[5], hi.z, lo.z);
    tm_split(x[6], x[7], hi.w, lo.w);
    const size_t o = xp_off(Npad, t, 8 * c);
    *reinterpret_cast<uint4*>(xp + o) = hi;
    *reinterpret_cast<uint4*>(xp + o + (size_t)64 * Npad) = lo;
    if (P.xsum) xp_sub_sum(P.xsum, Npad, t, c, x);
  }
  if (tid == 0) P.scale[t] = xp_pow2(e);
}

// 32 Q4_K weights of one row, columns j = 0..31 of a sub-block: the nibble at `sh` (0 or 4) of the
// 32 bytes W0, W1; w = ds*q - dm, as 16 hi and 16 lo words (column pairs 2m, 2m + 1).
__device__ __forceinline__ void tm_q4_row32(const uint4& W0, const uint4& W1, int sh, float ds, float dm,
                                            uint32_t (&h)[16], uint32_t (&l)[16]) {
  const uint32_t wd[8] = {W0.x, W0.y, W0.z, W0.w, W1.x, W1.y, W1.z, W1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t x = (wd[i] >> sh) & 0x0F0F0F0Fu;
    float w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) w[e] = fmaf(ds, __fsub_rn(tm_magic(x, e), 8388608.f), -dm);
    tm_split(w[0], w[1], h[2 * i], l[2 * i]);
    tm_split(w[2], w[3], h[2 * i + 1], l[2 * i + 1]);
  }
}
// 32 Q6_K weights of one row (columns j = 0..31 of a sub-block k of half h): low 4 bits from the
// ql bytes L0, L1 at shift ls, high 2 bits from the qh bytes H0, H1 at shift hs; scale ds0 for
// j < 16, ds1 for j >= 16; w = ds * (q - 32).
__device__ __forceinline__ void tm_q6_row32(const uint4& L0, const uint4& L1, const uint4& H0, const uint4& H1, int ls,
                                            int hs, float ds0, float ds1, uint32_t (&h)[16], uint32_t (&l)[16]) {
  const uint32_t lw[8] = {L0.x, L0.y, L0.z, L0.w, L1.x, L1.y, L1.z, L1.w};
  const uint32_t hw[8] = {H0.x, H0.y, H0.z, H0.w, H1.x, H1.y, H1.z, H1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t x = ((lw[i] >> ls) & 0x0F0F0F0Fu) | (((hw[i] >> hs) & 0x03030303u) << 4);
    const float ds = i < 4 ? ds0 : ds1;
    float w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) w[e] = __fmul_rn(ds, __fsub_rn(tm_magic(x, e), 8388640.f));
    tm_split(w[0], w[1], h[2 * i], l[2 * i]);
    tm_split(w[2], w[3], h[2 * i + 1], l[2 * i + 1]);
  }
}
// 32 Q4_K weights of one row in the exact form: q * sc as fp16 (q the nibble at `sh` of the 32
// bytes W0, W1; sc <= 63, so q * sc <= 945 is an integer fp16 holds exactly). The byte pair
// (q, 0x64) is the fp16 1024 + q; one fused multiply-add per two weights gives
// (1024 + q) * sc - 1024 sc with a single rounding of an exact integer result.
__device__ __forceinline__ void tm_q4_exact32(const uint4& W0, const uint4& W1, int sh, uint32_t sc, uint32_t (&a)[16]) {
  const __half2 s2 = __floats2half2_rn((float)sc, (float)sc);
  const __half2 c2 = __floats2half2_rn(-1024.f * (float)sc, -1024.f * (float)sc);
  const uint32_t wd[8] = {W0.x, W0.y, W0.z, W0.w, W1.x, W1.y, W1.z, W1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t x = (wd[i] >> sh) & 0x0F0F0F0Fu;
    uint32_t p0 = __byte_perm(x, 0x64u, 0x4140), p1 = __byte_perm(x, 0x64u, 0x4342);
    a[2 * i] = h2u(__hfma2(*reinterpret_cast<__half2*>(&p0), s2, c2));
    a[2 * i + 1] = h2u(__hfma2(*reinterpret_cast<__half2*>(&p1), s2, c2));
  }
}
// 8 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_st8(uint32_t taddr, const float (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
               "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
               : "memory");
}
// Two loads of 8 fp32 columns (at a and at b), one wait.
__device__ __forceinline__ void tc_ld8x2(uint32_t a, uint32_t b, float (&v)[8], float (&u)[8]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%16];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%17];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(a), "r"(b)
      : "memory");
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    v[e] = __uint_as_float(r[e]);
    u[e] = __uint_as_float(r[8 + e]);
  }
}

// Epilogue of one (row, token) value. lrow: row within the segment; vo: the value of row lrow ^ 1.
__device__ __forceinline__ void tm_epilogue(const TmmParams& P, const TmmSeg& S, int lrow, int tk, float v, float vo) {
  if (P.xscale) {   // undo the token's range scaling (a power of two: exact)
    const float sc = P.xscale[tk];
    v = __fmul_rn(v, sc);
    vo = __fmul_rn(vo, sc);
  }
  switch (S.epi) {
    case EPI_F32:
      S.out_f[(size_t)tk * P.out_ld + lrow] = v;
      break;
    case EPI_V: {
      const int kv = lrow / P.hd, d = lrow % P.hd;
      const int sq = P.B.seq ? P.B.seq[tk] : 0;
      S.out_h[((size_t)(sq * P.nkv + kv) * P.ctx + P.B.slot[tk]) * P.hd + d] = __float2half_rn(v);
    } break;
    case EPI_SWIGLU:   // rows (2i, 2i + 1) = (gate i, up i); fp32 [M][out_ld], packed by k_xpack_tok
      if ((lrow & 1) == 0) S.out_f[(size_t)tk * P.out_ld + (lrow >> 1)] = __fmul_rn(silu_f(v), vo);
      break;
    case EPI_ROPE_Q:
    case EPI_ROPE_K:   // rows (2i, 2i + 1) of a head = NeoX pair (i, i + hd/2)
      if ((lrow & 1) == 0) {
        const int hh = lrow / P.hd, i2 = (lrow % P.hd) >> 1, half = P.hd >> 1;
        const int rp = P.B.rpos[tk];
        const float cs = __ldg(P.cos_t + (size_t)rp * half + i2), sn = __ldg(P.sin_t + (size_t)rp * half + i2);
        const float o0 = __fsub_rn(__fmul_rn(v, cs), __fmul_rn(vo, sn));
        const float o1 = __fadd_rn(__fmul_rn(v, sn), __fmul_rn(vo, cs));
        if (S.epi == EPI_ROPE_Q) {
          float* q = S.out_f + (size_t)tk * P.out_ld + (size_t)hh * P.hd;
          q[i2] = o0;
          q[i2 + half] = o1;
        } else {
          const int sq = P.B.seq ? P.B.seq[tk] : 0;
          __half* dst = S.out_h + ((size_t)(sq * P.nkv + hh) * P.ctx + P.B.slot[tk]) * P.hd;
          dst[i2] = __float2half_rn(o0);
          dst[i2 + half] = __float2half_rn(o1);
        }
      }
      break;
  }
}

__global__ void __launch_bounds__(TM_THREADS, 1) k_tmm(const __grid_constant__ TmmParams P) {
  extern __shared__ uint8_t tm_dyn[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tm_dyn) + 1023) & ~(uintptr_t)1023);
  const int Npad = P.Npad;
  const uint32_t xbytes = 512u * (uint32_t)Npad;
  const int XS = P.xs;
  uint8_t* raw_ring = sm;
  uint8_t* x_ring = raw_ring + TM_RS * TM_RAW_BYTES;   // 1024-aligned (SWIZZLE_128B atoms)
  uint32_t* d_ring = reinterpret_cast<uint32_t*>(x_ring + (size_t)XS * xbytes);
  float* s_ring = reinterpret_cast<float*>(d_ring + TM_RS * TM_ROWS);   // [TM_SR][Npad][8]
  __shared__ __align__(8) uint64_t raw_full[TM_RS], raw_empty[TM_RS], a_full[TM_AS_MAX], sfree[TM_AS_MAX];
  __shared__ __align__(8) uint64_t x_full[TM_XS_MAX], x_free[TM_XS_MAX];
  __shared__ __align__(8) uint64_t acc_full, d_full[2], d_free[2], s_full[TM_SR], s_free[TM_SR];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort, s_last;
  volatile int* abort_f = &s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, sp = blockIdx.y;
  int si = 0;
  while (si + 1 < P.nseg && tile >= P.seg[si + 1].tile0) ++si;
  const TmmSeg& S = P.seg[si];
  const QView w = S.w;
  const int row0 = (tile - S.tile0) * TM_ROWS;
  const int G = P.G;
  const int g0 = (int)((long long)sp * G / P.nsplit), g1 = (int)((long long)(sp + 1) * G / P.nsplit);
  const int nsb = g1 - g0, nsub = 2 * nsb;
  const bool q4 = w.type == Q4K;
  // the exact form (this CTA's row tile): activation stages of a whole super-block, at least 2
  const bool ex = q4 && P.xsum != nullptr && Npad <= 64 && XS >= 4;
  const int XS2 = XS >> 1;
  const int rstride = q4 ? TM_RAW_Q4 : TM_RAW_Q6;
  const int AS = ex ? TM_XAS : tmm_as(Npad);
  const uint32_t acol = tmm_acol(Npad);

  if (threadIdx.x == 0) {
    for (int i = 0; i < TM_RS; ++i) { mbar_init(&raw_full[i], 32); mbar_init(&raw_empty[i], TM_DQ_WARPS); }
    for (int i = 0; i < AS; ++i) { mbar_init(&a_full[i], TM_DQ_WARPS); mbar_init(&sfree[i], 1); }
    for (int i = 0; i < XS; ++i) { mbar_init(&x_full[i], 1); mbar_init(&x_free[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&d_full[i], 1); mbar_init(&d_free[i], TM_DQ_WARPS); }
    for (int i = 0; i < TM_SR; ++i) { mbar_init(&s_full[i], 1); mbar_init(&s_free[i], TM_DQ_WARPS); }
    mbar_init(&acc_full, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&s_tmem, TM_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  pdl_trigger();
  if (threadIdx.x == 0) KQ_TRACE_AT(P.trace_id, 0);

  if (warp == 8) {
    // ---------------- raw loader: weights do not depend on the previous kernel (no PDL wait)
    const uint64_t pol = l2_evict_first_policy();
    // The nibble / ql and qh copies: lane = (row r8 of every 8-row tile, 16-byte chunk pc of a
    // 64-byte run). Every row this lane copies sits at position r8 of its tile (row0 is a
    // multiple of 128), so the row-dependent part of the address (row_plane_off) is a per-lane
    // base plus a multiple of the tile size, and per super-block only the swizzled column offset
    // changes.
    const int r8 = lane >> 2, pc = lane & 3;
    const size_t TB = tile_bytes(w.type, G);
    const uint8_t* pbase = w.base + (size_t)(row0 >> 3) * TB + (size_t)r8 * 128 * G;                    // p0, row r8
    const uint8_t* qbase = w.base + (size_t)(row0 >> 3) * TB + (size_t)8 * 128 * G + (size_t)r8 * 64 * G;   // Q6_K qh
    for (int k = 0; k < nsb; ++k) {
      const int slot = k % TM_RS;
      if (k >= TM_RS && !tm_wait(&raw_empty[slot], (uint32_t)((k / TM_RS) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f))
        break;
      const int g = g0 + k;
      uint8_t* dst = raw_ring + slot * TM_RAW_BYTES;
      const size_t o0 = p0_swz(r8, (size_t)g * 64 + pc * 16), o1 = p0_swz(r8, (size_t)64 * G + (size_t)g * 64 + pc * 16);
      const size_t oq = q6_qh_swz(G, r8, (size_t)g * 64 + pc * 16);
      // 8 rows per instruction, 4 lanes per 64-byte run
#pragma unroll 4
      for (int rb = 0; rb < TM_ROWS / 8; ++rb) {
        const int r = 8 * rb + r8, row = row0 + r;
        const bool ok = row < w.R;
        const uint8_t* tp = pbase + (size_t)rb * TB;
        cp_async16(dst + r * rstride + pc * 16, ok ? tp + o0 : w.base, ok ? 16u : 0u, pol);
        cp_async16(dst + r * rstride + 64 + pc * 16, ok ? tp + o1 : w.base, ok ? 16u : 0u, pol);
        if (!q4) cp_async16(dst + r * rstride + 128 + pc * 16, ok ? qbase + (size_t)rb * TB + oq : w.base, ok ? 16u : 0u, pol);
      }
      // Q4_K header / Q6_K scales (16 B per row); Q6_K d: the aligned 4-byte word that holds it
#pragma unroll
      for (int rb = 0; rb < TM_ROWS / 32; ++rb) {
        const int r = 32 * rb + lane, row = row0 + r;
        const bool ok = row < w.R;
        const uint8_t* src = ok ? w.base + row_plane_off(w.type, G, row, q4 ? 1 : 2, (size_t)g * 16) : w.base;
        cp_async16(dst + r * rstride + (q4 ? 128 : 192), src, ok ? 16u : 0u, pol);
        if (!q4) {
          const uintptr_t a = ok ? reinterpret_cast<uintptr_t>(w.base + row_plane_off(Q6K, G, row, 3, (size_t)g * 2))
                                 : reinterpret_cast<uintptr_t>(w.base);
          cp_async4(d_ring + slot * TM_ROWS + r, reinterpret_cast<const void*>(a & ~(uintptr_t)3), ok ? 4u : 0u);
        }
      }
      cp_async_arrive(&raw_full[slot]);
      if (lane == 0 && k == 0) KQ_TRACE_AT(P.trace_id, 1);
      if (lane == 0 && k == nsb - 1) KQ_TRACE_AT(P.trace_id, 11);
    }
    cp_async_wait_all();
  } else if (warp == 10) {
    // ---------------- activation loader
    if (lane == 0) {
      pdl_wait();
      KQ_TRACE_AT(P.trace_id, 8);
      const uint64_t pol = l2_evict_last_policy();
      int i = 0;
      if (ex) {
        // exact form: per super-block its sub-block sums, then its 4 activation groups in one copy
        int k = 0;
        for (; k < nsb; ++k) {
          const int ss = k % TM_SR, slot = k % XS2;
          if (k >= TM_SR && !tm_wait(&s_free[ss], (uint32_t)((k / TM_SR) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f))
            break;
          mbar_arrive_expect_tx(&s_full[ss], 32u * (uint32_t)Npad);
          bulk_g2s(s_ring + (size_t)ss * 8 * Npad, P.xsum + (size_t)(g0 + k) * 8 * Npad, 32u * (uint32_t)Npad, &s_full[ss], pol);
          if (k >= XS2 && !tm_wait(&x_free[slot], (uint32_t)((k / XS2) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f)) {
            ++k;
            break;
          }
          mbar_arrive_expect_tx(&x_full[slot], 2 * xbytes);
          bulk_g2s(x_ring + (size_t)slot * 2 * xbytes, P.xp + (size_t)(4 * (g0 + k)) * xp_group_halves(Npad), 2 * xbytes,
                   &x_full[slot], pol);
        }
        // drain: the last copy into each buffer has completed before the CTA exits
        for (int j = k - XS2 < 0 ? 0 : k - XS2; j < k; ++j)
          tm_wait(&x_full[j % XS2], (uint32_t)(j / XS2) & 1, P.err, KQ_DEV_ERR_DRAIN, abort_f);
        for (int j = k - TM_SR < 0 ? 0 : k - TM_SR; j < k; ++j)
          tm_wait(&s_full[j % TM_SR], (uint32_t)(j / TM_SR) & 1, P.err, KQ_DEV_ERR_DRAIN, abort_f);
        i = nsub;
      }
      for (; i < nsub && !ex; ++i) {
        const int slot = i % XS;
        if (i >= XS && !tm_wait(&x_free[slot], (uint32_t)((i / XS) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f))
          break;
        mbar_arrive_expect_tx(&x_full[slot], xbytes);
        bulk_g2s(x_ring + slot * xbytes, P.xp + (size_t)(4 * g0 + 2 * i) * xp_group_halves(Npad), xbytes, &x_full[slot], pol);
      }
      // drain: the last copy into each buffer has completed before the CTA exits
      if (!ex)
        for (int j = i - XS < 0 ? 0 : i - XS; j < i; ++j)
          tm_wait(&x_full[j % XS], (uint32_t)(j / XS) & 1, P.err, KQ_DEV_ERR_DRAIN, abort_f);
    }
  } else if (warp == 9) {
    // ---------------- MMA issue (one thread): A from tensor memory, activations from shared memory
    if (lane == 0 && ex) {
      // exact form: per super-block k one A stage (k & 1), one activation stage, and the
      // accumulator buffer k & 1, which the dequantising warps have read back (d_free) before it
      // is overwritten (accumulate = 0 at its first K step); 16 MMAs, three commits
      const uint32_t idesc = tc_idesc_f16(TM_ROWS, 2 * Npad);
      const uint64_t dX = sw128_desc(smem_u32(x_ring));
      const uint64_t gstep = (256u * (uint32_t)Npad) >> 4;
      for (int k = 0; k < nsb; ++k) {
        const int as = k & 1, xsl = k % XS2;
        if (!tm_spin(&a_full[as], (uint32_t)(k >> 1) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f)) break;
        if (!tm_spin(&x_full[xsl], (uint32_t)(k / XS2) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f)) break;
        if (k >= 2 && !tm_spin(&d_free[as], (uint32_t)((k >> 1) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f)) break;
        tc_fence_after();
        const uint32_t ta = tmem + TM_XA0 + (uint32_t)as * TM_XASTAGE_COLS, td = tmem + (uint32_t)as * TM_XD_COLS;
        const uint64_t x0 = dX + (uint64_t)(((uint32_t)xsl * 2 * xbytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)   // 16 K elements = 8 columns of A; 64-column group kk / 4, + 32 bytes per K step
          tc_mma_f16_ts(td, ta + 8 * kk, x0 + (kk >> 2) * gstep + 2 * (kk & 3), idesc, kk ? 1u : 0u);
        tc_commit(&sfree[as]);
        tc_commit(&x_free[xsl]);
        tc_commit(&d_full[as]);
        if (k == 0) KQ_TRACE_AT(P.trace_id, 3);
        if (k == nsb / 2) KQ_TRACE_AT(P.trace_id, 10);
      }
      KQ_TRACE_AT(P.trace_id, 5);
      tc_commit(&acc_full);
    } else if (lane == 0) {
      const uint32_t idesc1 = tc_idesc_f16(TM_ROWS, 2 * Npad), idesc2 = tc_idesc_f16(TM_ROWS, Npad);
      const uint64_t dX = sw128_desc(smem_u32(x_ring));
      for (int i = 0; i < nsub; ++i) {
        const int slot = i % AS, xsl = i % XS;
        if (!tm_wait(&a_full[slot], (uint32_t)(i / AS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f)) break;
        if (!tm_wait(&x_full[xsl], (uint32_t)(i / XS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f)) break;
        tc_fence_after();
        const uint32_t ta = tmem + acol + (uint32_t)slot * TM_ASTAGE_COLS;
        const uint64_t x0 = dX + (uint64_t)((xsl * xbytes) >> 4), gstep = (256u * (uint32_t)Npad) >> 4;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t ah = ta + 8 * kk, al = ah + 64;                     // 16 K elements = 8 columns
          const uint64_t bx = x0 + (kk >> 2) * gstep + 2 * (kk & 3);         // group, + 32 bytes per K step
          tc_mma_f16_ts(tmem, ah, bx, idesc1, (i | kk) ? 1u : 0u);          // hi(w) [hi(x); lo(x)]
          tc_mma_f16_ts(tmem + (uint32_t)Npad, al, bx, idesc2, 1u);          // + lo(w) hi(x)
        }
        tc_commit(&sfree[slot]);
        tc_commit(&x_free[xsl]);
        if (i == 0) KQ_TRACE_AT(P.trace_id, 3);
        if (i == nsub / 2) KQ_TRACE_AT(P.trace_id, 10);
      }
      KQ_TRACE_AT(P.trace_id, 5);
      tc_commit(&acc_full);   // also after a failure: arrives once the issued MMAs are done
    }
    __syncwarp();
  } else {
    // ---------------- dequantise (warps 0-7): lane = weight row 32 * (warp & 3) + lane (the warp's
    // TMEM lane quarter); warp >> 2 = which 64 of the sub-stage's 128 columns
    const int qd = warp & 3, hf = warp >> 2, r = 32 * qd + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
    bool ok = true;
    if (ex) {
      // ---------------- exact form. Per super-block k: the minimum term, the A stage (q * sc for
      // both halves of this warp's columns), then the read-back of super-block k - 1's buffer
      // scaled by its d into acc (this thread's row r, token half hf).
      // The minimum term -sum_b (dmin * mn_b) * xsum[t][b] is computed transposed: warp w takes the
      // tokens [w tpw, (w + 1) tpw) for the four rows lane + 32 j, so each sum loaded from shared
      // memory serves four rows (a quarter of the broadcast traffic of one row per thread); the
      // partial results stay in registers (mterm) and reach their owners once, at the end.
      const int nc = Npad >> 1, c0 = hf * nc, tpw = Npad >> 3, tw0 = warp * tpw;
      float acc[32], mterm[4][8];
#pragma unroll
      for (int e = 0; e < 32; ++e) acc[e] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) mterm[j][e] = 0.f;
      auto read_back = [&](int kb, float dk) -> bool {
        const int db = kb & 1;
        if (!__all_sync(0xffffffffu, tm_wait(&d_full[db], (uint32_t)(kb >> 1) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f)))
          return false;
        tc_fence_after();
        const uint32_t td = trow + (uint32_t)db * TM_XD_COLS;
#pragma unroll
        for (int cc = 0; cc < 32; cc += 8) {
          if (cc < nc) {
            float v[8], u[8];
            tc_ld8x2(td + (uint32_t)(c0 + cc), td + (uint32_t)(Npad + c0 + cc), v, u);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[cc + e] = __fmaf_rn(dk, __fadd_rn(v[e], u[e]), acc[cc + e]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_free[db]);
        return true;
      };
      float dprev = 0.f;
      for (int k = 0; k < nsb && ok; ++k) {
        const int slot = k % TM_RS, ss = k % TM_SR, as = k & 1;
        ok = __all_sync(0xffffffffu, tm_wait(&raw_full[slot], (uint32_t)(k / TM_RS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f));
        if (!ok) break;
        const uint8_t* rs = raw_ring + slot * TM_RAW_BYTES;
        ok = __all_sync(0xffffffffu, tm_wait(&s_full[ss], (uint32_t)(k / TM_SR) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f));
        if (!ok) break;
        {
          float dm[4][8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 Hj = lds128(rs + (lane + 32 * j) * rstride + 128);
            const float dmin = h2f_bits(Hj.x >> 16);
            const uint32_t mlo = Hj.z & 0x3F3F3F3Fu, mhi = ((Hj.w >> 4) & 0x0F0F0F0Fu) | ((Hj.z >> 2) & 0x30303030u);
#pragma unroll
            for (int b = 0; b < 8; ++b) dm[j][b] = __fmul_rn(dmin, (float)(((b < 4 ? mlo : mhi) >> (8 * (b & 3))) & 0xFFu));
          }
          const float4* xs4 = reinterpret_cast<const float4*>(s_ring + (size_t)ss * 8 * Npad + (size_t)tw0 * 8);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (e < tpw) {
              const float4 xa = xs4[2 * e], xb = xs4[2 * e + 1];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float u = __fmul_rn(dm[j][0], xa.x), w2 = __fmul_rn(dm[j][4], xb.x);
                u = __fmaf_rn(dm[j][1], xa.y, u); w2 = __fmaf_rn(dm[j][5], xb.y, w2);
                u = __fmaf_rn(dm[j][2], xa.z, u); w2 = __fmaf_rn(dm[j][6], xb.z, w2);
                u = __fmaf_rn(dm[j][3], xa.w, u); w2 = __fmaf_rn(dm[j][7], xb.w, w2);
                mterm[j][e] = __fadd_rn(mterm[j][e], __fadd_rn(u, w2));
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[ss]);
        // the A stage: this row's scales; both 128-column halves of the super-block
        const uint8_t* rw = rs + r * rstride;
        const uint4 H = lds128(rw + 128);
        const float d = h2f_bits(H.x & 0xFFFFu);
        const uint32_t sc_lo = H.y & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (H.w & 0x0F0F0F0Fu) | ((H.y >> 2) & 0x30303030u);
        if (k >= TM_XAS) {
          ok = __all_sync(0xffffffffu, tm_wait(&sfree[as], (uint32_t)((k >> 1) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f));
          if (!ok) break;
          tc_fence_after();   // the MMAs that read this stage have completed
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          // this warp's 64 columns of half h: sub-blocks 4h + 2hf (low nibbles), 4h + 2hf + 1 (high)
          const uint8_t* b = rw + hf * 64 + h * 32;
          const uint4 W0 = lds128(b), W1 = lds128(b + 16);
          const uint32_t scw = (h ? sc_hi : sc_lo) >> (16 * hf);
          uint32_t av[2][16];
          tm_q4_exact32(W0, W1, 0, scw & 0xFFu, av[0]);
          tm_q4_exact32(W0, W1, 4, (scw >> 8) & 0xFFu, av[1]);
          const uint32_t ta = trow + TM_XA0 + (uint32_t)as * TM_XASTAGE_COLS + 64u * (uint32_t)h + 32u * (uint32_t)hf;
          tc_st16(ta, av[0]);
          tc_st16(ta + 16, av[1]);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a_full[as]);
          mbar_arrive(&raw_empty[slot]);
        }
        if (warp == 0 && lane == 0 && k == 0) KQ_TRACE_AT(P.trace_id, 2);
        if (warp == 0 && lane == 0 && k == nsb / 2) KQ_TRACE_AT(P.trace_id, 9);
        if (warp == 0 && lane == 0 && k == nsb - 1) KQ_TRACE_AT(P.trace_id, 4);
        if (k >= 1) ok = read_back(k - 1, dprev);
        dprev = d;
      }
      if (ok) ok = read_back(nsb - 1, dprev);
      // the minimum terms to their owners through shared memory (the raw ring, read by nobody now:
      // every dequantising warp has passed its last super-block, every raw copy has landed)
      const bool all_ok = named_bar_and(2, TM_DQ_WARPS * 32, ok && !*abort_f);
      ok = all_ok;
      if (ok) {
        float* mbuf = reinterpret_cast<float*>(raw_ring);   // [128][Npad + 1]
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < tpw) mbuf[(lane + 32 * j) * (Npad + 1) + tw0 + e] = mterm[j][e];
        named_bar(2, TM_DQ_WARPS * 32);
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (e < nc) acc[e] = __fsub_rn(acc[e], mbuf[r * (Npad + 1) + c0 + e]);
        // the results into buffer 0 (read back already): value in column c, 0 in column Npad + c,
        // the form the shared epilogue reads
        const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int cc = 0; cc < 32; cc += 8) {
          if (cc < nc) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = acc[cc + e];
            tc_st8(trow + (uint32_t)(c0 + cc), v);
            tc_st8(trow + (uint32_t)(Npad + c0 + cc), z);
          }
        }
        tc_wait_st();
      }
    } else {
      for (int k = 0; k < nsb && ok; ++k) {
        const int slot = k % TM_RS;
        ok = __all_sync(0xffffffffu, tm_wait(&raw_full[slot], (uint32_t)(k / TM_RS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f));
        if (!ok) break;
        const uint8_t* rw = raw_ring + slot * TM_RAW_BYTES + r * rstride;
        // scales of this row for sub-stage h (columns 128h + 64hf + 32m + j):
        // Q4_K sub-block 4h + 2hf + m: (d*sc, dmin*mn); Q6_K sub-block k = 2hf + m: d*scale for j < 16, j >= 16
        float ds[2][2][2], dm[2][2];
        if (q4) {
          const uint4 H = lds128(rw + 128);
          const float d = h2f_bits(H.x & 0xFFFFu), dmin = h2f_bits(H.x >> 16);
          const uint32_t sc_lo = H.y & 0x3F3F3F3Fu, mn_lo = H.z & 0x3F3F3F3Fu;
          const uint32_t sc_hi = (H.w & 0x0F0F0F0Fu) | ((H.y >> 2) & 0x30303030u);
          const uint32_t mn_hi = ((H.w >> 4) & 0x0F0F0F0Fu) | ((H.z >> 2) & 0x30303030u);
  #pragma unroll
          for (int h = 0; h < 2; ++h)
  #pragma unroll
            for (int m = 0; m < 2; ++m) {
              const int sh = 8 * (2 * hf + m);   // sub-block 4h + 2hf + m: byte 2hf + m of word h
              ds[h][m][0] = ds[h][m][1] = __fmul_rn(d, (float)(((h ? sc_hi : sc_lo) >> sh) & 0xFFu));
              dm[h][m] = __fmul_rn(dmin, (float)(((h ? mn_hi : mn_lo) >> sh) & 0xFFu));
            }
        } else {
          const uint4 Sc = lds128(rw + 192);   // [u = 2h + jh][k]
          const uint32_t dw = d_ring[slot * TM_ROWS + r];
          const float d = h2f_bits(((r & 7) * G + g0 + k) & 1 ? dw >> 16 : dw & 0xFFFFu);
  #pragma unroll
          for (int h = 0; h < 2; ++h)
  #pragma unroll
            for (int m = 0; m < 2; ++m) {
              const int sh = 8 * (2 * hf + m);
              ds[h][m][0] = __fmul_rn(d, (float)(int8_t)(((h ? Sc.z : Sc.x) >> sh) & 0xFFu));
              ds[h][m][1] = __fmul_rn(d, (float)(int8_t)(((h ? Sc.w : Sc.y) >> sh) & 0xFFu));
              dm[h][m] = 0.f;
            }
        }
  #pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = 2 * k + h, as = i % AS;
          if (i >= AS) {
            ok = __all_sync(0xffffffffu, tm_wait(&sfree[as], (uint32_t)((i / AS) - 1) & 1, P.err, KQ_DEV_ERR_WAIT_EMPTY, abort_f));
            if (!ok) break;
            tc_fence_after();   // the MMAs that read this stage have completed
          }
          uint32_t hv[2][16], lv[2][16];
          if (q4) {
            // the 32 bytes of (h, c = hf): low nibbles = sub-block 4h + 2hf, high = 4h + 2hf + 1
            const uint8_t* b = rw + hf * 64 + h * 32;
            const uint4 W0 = lds128(b), W1 = lds128(b + 16);
            tm_q4_row32(W0, W1, 0, ds[h][0][0], dm[h][0], hv[0], lv[0]);
            tm_q4_row32(W0, W1, 4, ds[h][1][0], dm[h][1], hv[1], lv[1]);
          } else {
            // sub-block k = 2hf + m of half h: ql chunk c = m, nibble hf, qh shift 2k
            const uint8_t* hq = rw + 128 + h * 32;
            const uint4 H0 = lds128(hq), H1 = lds128(hq + 16);
  #pragma unroll
            for (int m = 0; m < 2; ++m) {
              const uint8_t* lq = rw + m * 64 + h * 32;
              tm_q6_row32(lds128(lq), lds128(lq + 16), H0, H1, 4 * hf, 2 * (2 * hf + m), ds[h][m][0], ds[h][m][1], hv[m], lv[m]);
            }
          }
          const uint32_t ta = trow + acol + (uint32_t)as * TM_ASTAGE_COLS + 32u * (uint32_t)hf;
          tc_st16(ta, hv[0]);
          tc_st16(ta + 16, hv[1]);
          tc_st16(ta + 64, lv[0]);
          tc_st16(ta + 80, lv[1]);
          tc_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[as]);
          if (warp == 0 && lane == 0 && i == 0) KQ_TRACE_AT(P.trace_id, 2);
          if (warp == 0 && lane == 0 && i == nsub / 2) KQ_TRACE_AT(P.trace_id, 9);
          if (warp == 0 && lane == 0 && i == nsub - 1) KQ_TRACE_AT(P.trace_id, 4);
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&raw_empty[slot]);
      }
    }
    // ---------------- epilogue (warps 0-7): TMEM lane quarter warp & 3, token half warp >> 2
    if (ok) ok = tm_wait(&acc_full, 0, P.err, KQ_DEV_ERR_WAIT_FULL, abort_f);
    const bool good = named_bar_and(1, TM_DQ_WARPS * 32, ok && !*abort_f);
    if (threadIdx.x == 0) KQ_TRACE_AT(P.trace_id, 6);
    if (good) {
      pdl_wait();
      tc_fence_after();
      const int q = warp & 3, rw_ = 32 * q + lane, lrow = row0 + rw_;
      const bool row_ok = lrow < w.R;
      const int nc = Npad / 2, c0 = (warp >> 2) * nc;
      const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
      const size_t Rtot = (size_t)P.ntiles * TM_ROWS, grow = (size_t)tile * TM_ROWS + rw_;
      if (P.nsplit > 1) {
        float* pp = P.part + (size_t)sp * Npad * Rtot + grow;
        for (int cc = 0; cc < nc; cc += 8) {
          float v[8], u[8];
          tc_ld8(tq + (uint32_t)(c0 + cc), v);
          tc_ld8(tq + (uint32_t)(Npad + c0 + cc), u);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (c0 + cc + e < P.M) __stcg(pp + (size_t)(c0 + cc + e) * Rtot, __fadd_rn(v[e], u[e]));
        }
        __threadfence();
        named_bar(1, TM_DQ_WARPS * 32);
        if (threadIdx.x == 0) s_last = atomicAdd(&P.ticket[tile], 1) == P.nsplit - 1;
        named_bar(1, TM_DQ_WARPS * 32);
        if (s_last) {
          __threadfence();
          // 8 tokens at a time: every split's partial requested before any is summed (one L2
          // round trip per group, not one per token and split); sums in split order
          for (int cb = 0; cb < nc; cb += 8) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = 0.f;
            for (int s2 = 0; s2 < P.nsplit; ++s2) {
              float u[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int tk = c0 + cb + e;
                u[e] = cb + e < nc && tk < P.M ? __ldcg(P.part + ((size_t)s2 * Npad + tk) * Rtot + grow) : 0.f;
              }
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], u[e]);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int tk = c0 + cb + e;
              const float vo = __shfl_xor_sync(0xffffffffu, v[e], 1);
              if (cb + e < nc && tk < P.M && row_ok) tm_epilogue(P, S, lrow, tk, v[e], vo);
            }
          }
          if (threadIdx.x == 0) P.ticket[tile] = 0;
        }
      } else {
        for (int cc = 0; cc < nc; cc += 8) {
          float v[8], u[8];
          tc_ld8(tq + (uint32_t)(c0 + cc), v);
          tc_ld8(tq + (uint32_t)(Npad + c0 + cc), u);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            v[e] = __fadd_rn(v[e], u[e]);
            const float vo = __shfl_xor_sync(0xffffffffu, v[e], 1);
            if (c0 + cc + e < P.M && row_ok) tm_epilogue(P, S, lrow, c0 + cc + e, v[e], vo);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) KQ_TRACE_AT(P.trace_id, 7);
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, TM_TMEM_COLS);
  }
}

}  // namespace kq
