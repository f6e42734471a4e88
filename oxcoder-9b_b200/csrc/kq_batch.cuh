// kq_batch.cuh -- the non-GEMM kernels of a forward pass over M <= 128 tokens at once (the
// verification pass over a draft tree, a prefill chunk); the GEMMs are k_tmm (kq_tmm.cuh).
//
//  * k_bnorm: per token, the residual add and fp64-sum RMS norm (or the embedding row), writing
//    h and the packed hi/lo fp16 input of the next GEMM.
//  * k_battn: attention of every token of the pass over the cache prefix and the tree slots, with
//    each token's ancestor mask. Flash-style on the tensor cores (mma.sync m16n8k16, fp32
//    accumulation): a warp owns 16 query rows (token x head of one KV group), the CTA streams
//    blocks of 64 keys of one KV head through shared memory (cp.async, two stages), the scores
//    S = Q K^T take Q as hi + lo fp16 (K is fp16 in the cache, exact), the online softmax runs in
//    fp32 registers and O += P V takes P as hi + lo fp16 (V exact). Key ranges are split over
//    CTAs; the last CTA of each (KV head, row group) merges the partials in split order.
//  * k_argmax_rows: per-token argmax of the logits.
#pragma once
#include "kq_common.cuh"
#include "kq_qformat.cuh"
#include "kq_gemv.cuh"
#include "kq_tmm.cuh"
#include <cfloat>

namespace kq {

constexpr int MM_MAXM = 128;           // tokens per batched pass (verification, prefill)

// ------------------------------------------------------------------------------ norm / embedding
struct BNormParams {
  int M, D;
  const int* tok;          // [M] (embedding mode)
  QView emb;               // embedding matrix, or type 0: residual mode
  float* h;                // [M][D] residual stream (read-modify-write)
  const float* y;          // [M][D] block output to add (residual mode), or null
  const float* gamma;      // [D]
  float eps;
  __half* xp;              // packed input of the next GEMM (C = D)
  float* xscale;           // [M] the power of two each packed row was divided by (xp_scale_exp)
  float* xsum;             // sub-block sums of the packed rows (xp_sub_sum; D % 256 == 0), or null
  int Npad;
  int vocab;
  int* err;
};
constexpr int BN_THREADS = 512;
// One CTA per token; thread t owns the 8-column chunks t, t + 512, ... (float4 loads, and one
// 16-byte hi and one 16-byte lo store of the packed layout per chunk).
__global__ void __launch_bounds__(BN_THREADS) k_bnorm(const __grid_constant__ BNormParams P) {
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ double red[BN_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  float* h = P.h + (size_t)t * P.D;
  int tok = 0;
  if (P.emb.base) {
    tok = P.tok[t];
    if (tok < 0 || tok >= P.vocab) {
      if (tid == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_TOKEN);
      tok = 0;
    }
  }
  double acc = 0.0;
  float hmax = 0.f, gmax = 0.f;   // bound of the output row: max|h| * s * max|gamma|
  const int nch = P.D / 8;
  for (int c = tid; c < nch; c += BN_THREADS) {
    float v[8];
    if (P.emb.base) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = dequant_elem(P.emb, tok, 8 * c + e);
    } else {
      const float4 a0 = reinterpret_cast<const float4*>(h)[2 * c], a1 = reinterpret_cast<const float4*>(h)[2 * c + 1];
      v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
      if (P.y) {
        const float4* y4 = reinterpret_cast<const float4*>(P.y + (size_t)t * P.D);
        const float4 b0 = y4[2 * c], b1 = y4[2 * c + 1];
        v[0] = __fadd_rn(v[0], b0.x); v[1] = __fadd_rn(v[1], b0.y); v[2] = __fadd_rn(v[2], b0.z); v[3] = __fadd_rn(v[3], b0.w);
        v[4] = __fadd_rn(v[4], b1.x); v[5] = __fadd_rn(v[5], b1.y); v[6] = __fadd_rn(v[6], b1.z); v[7] = __fadd_rn(v[7], b1.w);
      }
    }
    reinterpret_cast<float4*>(h)[2 * c] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(h)[2 * c + 1] = make_float4(v[4], v[5], v[6], v[7]);
    const float4 g0 = reinterpret_cast<const float4*>(P.gamma)[2 * c], g1 = reinterpret_cast<const float4*>(P.gamma)[2 * c + 1];
    gmax = fmaxf(gmax, fmaxf(fmaxf(fmaxf(fabsf(g0.x), fabsf(g0.y)), fmaxf(fabsf(g0.z), fabsf(g0.w))),
                             fmaxf(fmaxf(fabsf(g1.x), fabsf(g1.y)), fmaxf(fabsf(g1.z), fabsf(g1.w)))));
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      acc = __dadd_rn(acc, __dmul_rn((double)v[e], (double)v[e]));
      hmax = fmaxf(hmax, fabsf(v[e]));
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    acc += __shfl_xor_sync(0xffffffffu, acc, off);
    hmax = fmaxf(hmax, __shfl_xor_sync(0xffffffffu, hmax, off));
    gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, off));
  }
  __shared__ float redm[2][BN_THREADS / 32];
  if (lane == 0) { red[warp] = acc; redm[0][warp] = hmax; redm[1][warp] = gmax; }
  __syncthreads();
  double tot = 0.0;
  for (int w = 0; w < BN_THREADS / 32; ++w) {
    tot += red[w];
    hmax = fmaxf(hmax, redm[0][w]);
    gmax = fmaxf(gmax, redm[1][w]);
  }
  const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__double2float_rn(tot / (double)P.D), P.eps)));
  // every output |fl(fl(h s) gamma)| <= hmax * s * gmax (1 + 2^-22); the slack covers the roundings
  const int e_t = xp_scale_exp(__fmul_rn(__fmul_rn(__fmul_rn(hmax, s), gmax), 1.0000005f));
  const float inv = xp_pow2(-e_t);
  if (tid == 0) P.xscale[t] = xp_pow2(e_t);
  for (int c = tid; c < nch; c += BN_THREADS) {
    const float4 a0 = reinterpret_cast<const float4*>(h)[2 * c], a1 = reinterpret_cast<const float4*>(h)[2 * c + 1];
    const float4 g0 = reinterpret_cast<const float4*>(P.gamma)[2 * c], g1 = reinterpret_cast<const float4*>(P.gamma)[2 * c + 1];
    float x[8] = {__fmul_rn(__fmul_rn(a0.x, s), g0.x), __fmul_rn(__fmul_rn(a0.y, s), g0.y),
                  __fmul_rn(__fmul_rn(a0.z, s), g0.z), __fmul_rn(__fmul_rn(a0.w, s), g0.w),
                  __fmul_rn(__fmul_rn(a1.x, s), g1.x), __fmul_rn(__fmul_rn(a1.y, s), g1.y),
                  __fmul_rn(__fmul_rn(a1.z, s), g1.z), __fmul_rn(__fmul_rn(a1.w, s), g1.w)};
    if (e_t) {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __fmul_rn(x[e], inv);
    }
    uint4 hi, lo;
    tm_split(x[0], x[1], hi.x, lo.x);
    tm_split(x[2], x[3], hi.y, lo.y);
    tm_split(x[4], x[5], hi.z, lo.z);
    tm_split(x[6], x[7], hi.w, lo.w);
    const size_t o = xp_off(P.Npad, t, 8 * c);   // 8 consecutive halves
    *reinterpret_cast<uint4*>(P.xp + o) = hi;
    *reinterpret_cast<uint4*>(P.xp + o + (size_t)64 * P.Npad) = lo;
    if (P.xsum) xp_sub_sum(P.xsum, P.Npad, t, c, x);   // whole warps: nch is a multiple of 32
  }
}

// ------------------------------------------------------------------------------ tree attention
constexpr int BA_KB = 64;                   // keys per block
constexpr int BA_WARPS = 4;                 // warps per CTA, 16 query rows each
constexpr int BA_ROWS = 16 * BA_WARPS;      // query rows (token x head) per CTA
constexpr int BA_LD = 128 + 8;              // padded shared-memory row (halves): conflict-free
constexpr size_t BA_SMEM = (size_t)2 * 2 * BA_KB * BA_LD * 2;   // K and V blocks, two stages
constexpr int BA_PLD = 128 + 4;             // partial row: o[128], m, l, padding (16-byte rows)
constexpr int BA_MAX_SPLIT = 32;

struct BAttnParams {
  const float* q;                    // [M][NH * HD] rotated queries
  const __half* kc;                  // [n_kv][ctx][HD]
  const __half* vc;
  __half* out_xp;                    // packed input of the o GEMM (C = NH * HD)
  int Npad;
  BatchParams B;
  int n_kv, ctx, npos;               // keys [0, npos) may be attended
  float scale;
  int nsplit, nblk;                  // key blocks per split
  float* part;                       // [n_kv][rowgroups][nsplit][BA_ROWS][BA_PLD]
  int* ticket;                       // [n_kv][rowgroups]
};

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void cp_async16_plain(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// CTA (KV head, row group of BA_ROWS query rows, key split). Query row qr = token * G + head.
template <int G>
__global__ void __launch_bounds__(BA_WARPS * 32) k_battn(const __grid_constant__ BAttnParams P) {
  constexpr int HD = 128;
  extern __shared__ __align__(16) uint8_t ba_sm[];
  __half* ksm = reinterpret_cast<__half*>(ba_sm);    // [2][BA_KB][BA_LD]
  __half* vsm = ksm + 2 * BA_KB * BA_LD;
  __shared__ int s_last;
  const int kv = blockIdx.x, rg = blockIdx.y, sp = blockIdx.z, rowgroups = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, grp = lane >> 2, t4 = lane & 3;
  const int M = P.B.M, nrows = M * G, tbase = P.B.tree_base;
  const int ra = rg * BA_ROWS + warp * 16 + grp, rb = ra + 8;
  const int nblocks = (P.npos + BA_KB - 1) / BA_KB;
  const int b_begin = sp * P.nblk, b_end = min(b_begin + P.nblk, nblocks);
  const int NHHD = P.n_kv * G * HD;
  pdl_wait();
  pdl_trigger();
  const __half* kg = P.kc + (size_t)kv * P.ctx * HD;
  const __half* vg = P.vc + (size_t)kv * P.ctx * HD;
  auto load_block = [&](int b, int stage) {
    __half* kd = ksm + stage * BA_KB * BA_LD;
    __half* vd = vsm + stage * BA_KB * BA_LD;
    for (int i = tid; i < BA_KB * 16; i += BA_WARPS * 32) {   // 16 chunks of 16 B per key row
      const int r = i >> 4, c = i & 15, t = b * BA_KB + r;
      const bool ok = t < P.npos;
      const size_t off = (size_t)(ok ? t : 0) * HD + c * 8;
      cp_async16_plain(kd + r * BA_LD + c * 8, kg + off, ok ? 16u : 0u);
      cp_async16_plain(vd + r * BA_LD + c * 8, vg + off, ok ? 16u : 0u);
    }
  };
  if (b_begin < b_end) load_block(b_begin, 0);
  cp_async_commit();

  // Q fragments (hi / lo) of rows ra (a0, a2) and rb (a1, a3)
  const bool va = ra < nrows, vb = rb < nrows;
  const int ta = va ? ra / G : 0, tb = vb ? rb / G : 0;
  const float* qa = P.q + (size_t)ta * NHHD + (size_t)(kv * G + ra % G) * HD;
  const float* qb = P.q + (size_t)tb * NHHD + (size_t)(kv * G + rb % G) * HD;
  uint32_t qh[8][4], ql[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int d = 16 * ks + 2 * t4;
    const float2 z = make_float2(0.f, 0.f);
    const float2 x0 = va ? *reinterpret_cast<const float2*>(qa + d) : z;
    const float2 x1 = vb ? *reinterpret_cast<const float2*>(qb + d) : z;
    const float2 x2 = va ? *reinterpret_cast<const float2*>(qa + d + 8) : z;
    const float2 x3 = vb ? *reinterpret_cast<const float2*>(qb + d + 8) : z;
    tm_split(x0.x, x0.y, qh[ks][0], ql[ks][0]);
    tm_split(x1.x, x1.y, qh[ks][1], ql[ks][1]);
    tm_split(x2.x, x2.y, qh[ks][2], ql[ks][2]);
    tm_split(x3.x, x3.y, qh[ks][3], ql[ks][3]);
  }
  const unsigned long long ma0 = va ? P.B.mask[2 * ta] : ~0ull, ma1 = va ? P.B.mask[2 * ta + 1] : ~0ull;
  const unsigned long long mb0 = vb ? P.B.mask[2 * tb] : ~0ull, mb1 = vb ? P.B.mask[2 * tb + 1] : ~0ull;

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  const int mi = lane >> 3;
  for (int b = b_begin; b < b_end; ++b) {
    const int st = (b - b_begin) & 1;
    if (b + 1 < b_end) load_block(b + 1, st ^ 1);
    cp_async_commit();
    cp_async_wait1();
    __syncthreads();
    const __half* kd = ksm + st * BA_KB * BA_LD;
    const __half* vd = vsm + st * BA_KB * BA_LD;
    // ---- S = Q K^T (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4(kd + (16 * np + ((mi >> 1) << 3) + (lane & 7)) * BA_LD + 16 * ks + ((mi & 1) << 3), r0, r1, r2, r3);
        mma16816(s[2 * np], ql[ks], r0, r1);
        mma16816(s[2 * np], qh[ks], r0, r1);
        mma16816(s[2 * np + 1], ql[ks], r2, r3);
        mma16816(s[2 * np + 1], qh[ks], r2, r3);
      }
    }
    // ---- scale, mask, online softmax (rows ra: elements 0-1, rb: elements 2-3)
    const int t0 = b * BA_KB;
    const bool full = t0 + BA_KB <= min(P.npos, tbase);
    float bmA = -INFINITY, bmB = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float a = __fmul_rn(s[n][e], P.scale);
        if (!full) {
          const int t = t0 + 8 * n + 2 * t4 + (e & 1);
          const bool vis = t < P.npos && (e < 2 ? slot_attended(t, tbase, ma0, ma1) : slot_attended(t, tbase, mb0, mb1));
          if (!vis) a = -INFINITY;
        }
        s[n][e] = a;
        if (e < 2) bmA = fmaxf(bmA, a); else bmB = fmaxf(bmB, a);
      }
    }
    bmA = fmaxf(bmA, __shfl_xor_sync(0xffffffffu, bmA, 1));
    bmA = fmaxf(bmA, __shfl_xor_sync(0xffffffffu, bmA, 2));
    bmB = fmaxf(bmB, __shfl_xor_sync(0xffffffffu, bmB, 1));
    bmB = fmaxf(bmB, __shfl_xor_sync(0xffffffffu, bmB, 2));
    const float nmA = fmaxf(mA, bmA), nmB = fmaxf(mB, bmB);
    const float uA = nmA == -INFINITY ? 0.f : nmA, uB = nmB == -INFINITY ? 0.f : nmB;
    const float fA = expf(__fsub_rn(mA, uA)), fB = expf(__fsub_rn(mB, uB));
    mA = nmA;
    mB = nmB;
    float sA = 0.f, sB = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = expf(__fsub_rn(s[n][e], e < 2 ? uA : uB));
        s[n][e] = p;
        if (e < 2) sA = __fadd_rn(sA, p); else sB = __fadd_rn(sB, p);
      }
    }
    sA = __fadd_rn(sA, __shfl_xor_sync(0xffffffffu, sA, 1));
    sA = __fadd_rn(sA, __shfl_xor_sync(0xffffffffu, sA, 2));
    sB = __fadd_rn(sB, __shfl_xor_sync(0xffffffffu, sB, 1));
    sB = __fadd_rn(sB, __shfl_xor_sync(0xffffffffu, sB, 2));
    lA = fmaf(lA, fA, sA);
    lB = fmaf(lB, fB, sB);
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= fA; o[n][1] *= fA; o[n][2] *= fB; o[n][3] *= fB;
    }
    // ---- O += P V
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t ah[4], al[4];
      tm_split(s[2 * j][0], s[2 * j][1], ah[0], al[0]);
      tm_split(s[2 * j][2], s[2 * j][3], ah[1], al[1]);
      tm_split(s[2 * j + 1][0], s[2 * j + 1][1], ah[2], al[2]);
      tm_split(s[2 * j + 1][2], s[2 * j + 1][3], ah[3], al[3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vd + (16 * j + ((mi & 1) << 3) + (lane & 7)) * BA_LD + 16 * dp + ((mi >> 1) << 3), r0, r1, r2, r3);
        mma16816(o[2 * dp], al, r0, r1);
        mma16816(o[2 * dp], ah, r0, r1);
        mma16816(o[2 * dp + 1], al, r2, r3);
        mma16816(o[2 * dp + 1], ah, r2, r3);
      }
    }
    __syncthreads();   // the stage is refilled by the next iteration's prefetch
  }
  // ---- partial (o, m, l) of this split: [kv][rg][sp][BA_ROWS][BA_PLD]
  const size_t pbase = (((size_t)kv * rowgroups + rg) * P.nsplit + sp) * BA_ROWS * BA_PLD;
  float* pa = P.part + pbase + (size_t)(warp * 16 + grp) * BA_PLD;
  float* pb = pa + 8 * BA_PLD;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    __stcg(reinterpret_cast<float2*>(pa + 8 * n + 2 * t4), make_float2(o[n][0], o[n][1]));
    __stcg(reinterpret_cast<float2*>(pb + 8 * n + 2 * t4), make_float2(o[n][2], o[n][3]));
  }
  if (t4 == 0) {
    __stcg(pa + HD, mA); __stcg(pa + HD + 1, lA);
    __stcg(pb + HD, mB); __stcg(pb + HD + 1, lB);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&P.ticket[kv * rowgroups + rg], 1) == P.nsplit - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- merge the splits in order: per-row weights exp(m_s - max) and the sum L first, then
  // float4 columns (the K/V stages are free: their copies all completed in the loop)
  float* fac = reinterpret_cast<float*>(ba_sm);   // [nsplit][BA_ROWS]
  float* lsum = fac + P.nsplit * BA_ROWS;         // [BA_ROWS]
  const float* mbp = P.part + ((size_t)kv * rowgroups + rg) * P.nsplit * BA_ROWS * BA_PLD;
  if (tid < BA_ROWS) {
    float Mx = -INFINITY;
    for (int s2 = 0; s2 < P.nsplit; ++s2) Mx = fmaxf(Mx, __ldcg(mbp + ((size_t)s2 * BA_ROWS + tid) * BA_PLD + HD));
    float L = 0.f;
    for (int s2 = 0; s2 < P.nsplit; ++s2) {
      const float* pr = mbp + ((size_t)s2 * BA_ROWS + tid) * BA_PLD;
      const float ms = __ldcg(pr + HD);
      const float wgt = ms == -INFINITY ? 0.f : expf(__fsub_rn(ms, Mx));
      fac[s2 * BA_ROWS + tid] = wgt;
      L = fmaf(wgt, __ldcg(pr + HD + 1), L);
    }
    lsum[tid] = L;
  }
  __syncthreads();
  for (int e = tid; e < BA_ROWS * (HD / 4); e += BA_WARPS * 32) {
    const int lr = e / (HD / 4), d4 = e % (HD / 4), qr = rg * BA_ROWS + lr;
    if (qr >= nrows) break;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int s2 = 0; s2 < P.nsplit; ++s2) {
      const float wgt = fac[s2 * BA_ROWS + lr];
      const float4 v = __ldcg(reinterpret_cast<const float4*>(mbp + ((size_t)s2 * BA_ROWS + lr) * BA_PLD) + d4);
      O.x = fmaf(wgt, v.x, O.x); O.y = fmaf(wgt, v.y, O.y); O.z = fmaf(wgt, v.z, O.z); O.w = fmaf(wgt, v.w, O.w);
    }
    const float L = lsum[lr];
    const int col = (kv * G + qr % G) * HD + 4 * d4, tk = qr / G;
    xp_store(P.out_xp, P.Npad, tk, col, __fdiv_rn(O.x, L));
    xp_store(P.out_xp, P.Npad, tk, col + 1, __fdiv_rn(O.y, L));
    xp_store(P.out_xp, P.Npad, tk, col + 2, __fdiv_rn(O.z, L));
    xp_store(P.out_xp, P.Npad, tk, col + 3, __fdiv_rn(O.w, L));
  }
  if (tid == 0) P.ticket[kv * rowgroups + rg] = 0;
}

// Per-token argmax of the logits (lowest index on ties), one CTA per token.
__global__ void __launch_bounds__(256) k_argmax_rows(const float* logits, int V, int* out) {
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float bv[8];
  __shared__ int bi[8];
  pdl_wait();
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

// ------------------------------------------------------------------------------ batched decode attention
// One token per sequence, each over its own sequence's cache (batched decode of many sequences):
// CTA = (token, KV head, split of positions [0, pos + 1)); 4 warps take positions in turn, a lane
// owns 4 of the 128 dims, the G query heads' scores are warp sums (xor tree), online softmax per
// warp, the warps' (m, l, o) combined in fixed order into the split's partial. fp32 throughout,
// fp16 K/V as stored. k_dattn_merge merges the splits in order into the packed o-GEMM input.
constexpr int DA_WARPS = 4;
constexpr int DA_MAX_SPLIT = 64;   // key splits (64 keys each for the single-token step at ctx 4K;
                                   // measured against 16 / 32 / 48 / 96 / 128: 64 is fastest)
struct DAttnParams {
  const float* q;            // [M][NH_l * HD] rotated queries
  const __half* kc;          // [nseq][n_kv][ctx][HD]
  const __half* vc;
  const int* seq;            // [M] sequence of each token
  const int* pos;            // [M] its position (attends to [0, pos])
  int n_kv, ctx, nsplit;
  float scale;
  float* part;               // [M][n_kv][nsplit][G][HD + 4] (o, m, l, pad)
  __half* out_xp;            // packed o-GEMM input (merge), or
  float* out_f;              // fp32 [M][n_kv * G * HD] (the decode step's GEMV input)
  int Npad;
  const DecodeState* st;     // decode step (M = 1): position, tree base and ancestor mask from the
                             // device-resident step state instead of pos / seq
  int* err;
  int trace_id;              // launch index for the optional phase trace (KQ_TRACE builds)
};
template <int G>
__global__ void __launch_bounds__(DA_WARPS * 32) k_dattn(const __grid_constant__ DAttnParams P) {
  constexpr int HD = 128, PLD = HD + 4;
  const int t = blockIdx.x, kv = blockIdx.y, sp = blockIdx.z, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float s_m[DA_WARPS][G], s_l[DA_WARPS][G];
  __shared__ __align__(16) float s_o[DA_WARPS][G][HD];
  pdl_wait();
  pdl_trigger();
  const int n = P.pos[t] + 1, per = (n + P.nsplit - 1) / P.nsplit;
  const int p0 = min(n, sp * per), p1 = min(n, p0 + per);
  const size_t cbase = ((size_t)P.seq[t] * P.n_kv + kv) * P.ctx * HD;
  const __half* kb = P.kc + cbase;
  const __half* vb = P.vc + cbase;
  const int NHHD = P.n_kv * G * HD;
  float q[G][4], o[G][4], m[G], l[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float4 qq = *reinterpret_cast<const float4*>(P.q + (size_t)t * NHHD + (size_t)(kv * G + g) * HD + 4 * lane);
    q[g][0] = qq.x; q[g][1] = qq.y; q[g][2] = qq.z; q[g][3] = qq.w;
    o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
    m[g] = -INFINITY;
    l[g] = 0.f;
  }
  for (int p = p0 + warp; p < p1; p += DA_WARPS) {
    const uint2 kr = __ldcs(reinterpret_cast<const uint2*>(kb + (size_t)p * HD) + lane);
    const uint2 vr = __ldcs(reinterpret_cast<const uint2*>(vb + (size_t)p * HD) + lane);
    const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kr.x));
    const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kr.y));
    const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vr.x));
    const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vr.y));
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float d = __fmul_rn(q[g][0], k01.x);
      d = __fmaf_rn(q[g][1], k01.y, d);
      d = __fmaf_rn(q[g][2], k23.x, d);
      d = __fmaf_rn(q[g][3], k23.y, d);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, off));
      const float sc = __fmul_rn(d, P.scale);
      const float mn = fmaxf(m[g], sc);
      const float f = expf(__fsub_rn(m[g], mn)), e = expf(__fsub_rn(sc, mn));
      m[g] = mn;
      l[g] = __fmaf_rn(l[g], f, e);
      o[g][0] = __fmaf_rn(o[g][0], f, __fmul_rn(e, v01.x));
      o[g][1] = __fmaf_rn(o[g][1], f, __fmul_rn(e, v01.y));
      o[g][2] = __fmaf_rn(o[g][2], f, __fmul_rn(e, v23.x));
      o[g][3] = __fmaf_rn(o[g][3], f, __fmul_rn(e, v23.y));
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) { s_m[warp][g] = m[g]; s_l[warp][g] = l[g]; }
    *reinterpret_cast<float4*>(&s_o[warp][g][4 * lane]) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
  }
  __syncthreads();
  // the warps' partials combined in warp order: thread = (head g, 4 dims)
  float* part = P.part + (((size_t)t * P.n_kv + kv) * P.nsplit + sp) * G * PLD;
  for (int e = threadIdx.x; e < G * (HD / 4); e += DA_WARPS * 32) {
    const int g = e / (HD / 4), d4 = e % (HD / 4);
    float M = -INFINITY;
    for (int w = 0; w < DA_WARPS; ++w) M = fmaxf(M, s_m[w][g]);
    float L = 0.f, O0 = 0.f, O1 = 0.f, O2 = 0.f, O3 = 0.f;
    for (int w = 0; w < DA_WARPS; ++w) {
      const float wt = s_m[w][g] == -INFINITY ? 0.f : expf(__fsub_rn(s_m[w][g], M));
      const float4 ow = *reinterpret_cast<const float4*>(&s_o[w][g][4 * d4]);
      L = __fmaf_rn(wt, s_l[w][g], L);
      O0 = __fmaf_rn(wt, ow.x, O0); O1 = __fmaf_rn(wt, ow.y, O1); O2 = __fmaf_rn(wt, ow.z, O2); O3 = __fmaf_rn(wt, ow.w, O3);
    }
    __stcg(reinterpret_cast<float4*>(part + (size_t)g * PLD) + d4, make_float4(O0, O1, O2, O3));
    if (d4 == 0) { __stcg(part + (size_t)g * PLD + HD, M); __stcg(part + (size_t)g * PLD + HD + 1, L); }
  }
}
// Tensor-core form: one warp per (token, KV head, split); 32-key blocks of K/V through shared
// memory (cp.async, two stages, padded rows); the G query heads are rows 0..G-1 of an m16 tile
// (Q as hi + lo fp16), S = Q K^T and O += P V on mma.sync with fp32 accumulation and the online
// softmax in registers, as the tree attention. Same partial layout as k_dattn (k_dattn_merge).
// Decode step (P.st): the preceding q/k/v GEMV writes only cache slot pos; every older slot was
// written by an earlier step (hundreds of launches back), so the first two blocks are requested
// before the dependency wait when none of their keys is pos, and the K/V stream overlaps the
// GEMV's tail. The step state (pos, tree) was written by the previous step's output head.
constexpr int DM_KB = 32;                                            // keys per block
constexpr size_t DM_SMEM = (size_t)2 * 2 * DM_KB * BA_LD * 2;          // K and V, two stages
// One warp's flash pass (token t, KV head kv, keys [0, n) attended): the 32-key blocks starting at
// p0, p0 + bs, p0 + 2 bs, ... below p1 through its two shared-memory stages ksm / vsm; returns the
// unnormalised output rows and the running max / sum of rows grp (A) and grp + 8 (B). With a
// decode step state (P.st) the first two blocks are requested before the dependency wait when
// none of their keys is the new slot pos; the wait is always taken in that case.
template <int G>
__device__ __forceinline__ void dm_warp_pass(const DAttnParams& P, int t, int kv, int n, int p0, int bs, int p1,
                                             __half* ksm, __half* vsm, float (&o)[16][4], float& mA, float& mB,
                                             float& lA, float& lB) {
  constexpr int HD = 128;
  const int lane = threadIdx.x & 31, grp = lane >> 2, t4 = lane & 3;
  const int tbase = P.st ? P.st->tree_base : n;
  const unsigned long long tm0 = P.st ? P.st->mask[0] : 0ull, tm1 = P.st ? P.st->mask[1] : 0ull;
  const size_t cbase = ((size_t)(P.seq ? P.seq[t] : 0) * P.n_kv + kv) * P.ctx * HD;
  const __half* kg = P.kc + cbase;
  const __half* vg = P.vc + cbase;
  auto load_block = [&](int b0, int stage) {
    __half* kd = ksm + stage * DM_KB * BA_LD;
    __half* vd = vsm + stage * DM_KB * BA_LD;
#pragma unroll 4
    for (int i = lane; i < DM_KB * 16; i += 32) {   // 16 chunks of 16 B per key row
      const int r = i >> 4, c = i & 15, tk = b0 + r;
      const bool ok = tk < p1;
      const size_t off = (size_t)(ok ? tk : b0) * HD + c * 8;
      cp_async16_plain(kd + r * BA_LD + c * 8, kg + off, ok ? 16u : 0u);
      cp_async16_plain(vd + r * BA_LD + c * 8, vg + off, ok ? 16u : 0u);
    }
  };
  // blocks 0 and 1 before the wait (decode step, keys all below pos); cp.async groups are
  // committed in the same places either way, and wait_group 1 below only ever waits for more
  bool pre0 = false, pre1 = false;
  if (P.st) {
    pre0 = p0 < p1 && min(p0 + DM_KB, p1) <= n - 1;
    pre1 = p0 + bs < p1 && min(p0 + bs + DM_KB, p1) <= n - 1;
    if (pre0) load_block(p0, 0);
    cp_async_commit();
    if (pre1) load_block(p0 + bs, 1);
    cp_async_commit();
    pdl_wait();
    if (lane == 0) KQ_TRACE_AT(P.trace_id, 1);
  }
  if (p0 < p1 && !pre0) load_block(p0, 0);
  cp_async_commit();
  // Q fragments: rows grp (a0, a2) and grp + 8 (a1, a3); rows >= G are zero
  const int NHHD = P.n_kv * G * HD;
  const bool va = grp < G, vb = grp + 8 < G;
  const float* qa = P.q + (size_t)t * NHHD + (size_t)(kv * G + (va ? grp : 0)) * HD;
  const float* qb = P.q + (size_t)t * NHHD + (size_t)(kv * G + (vb ? grp + 8 : 0)) * HD;
  uint32_t qh[8][4], ql[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int d = 16 * ks + 2 * t4;
    const float2 z = make_float2(0.f, 0.f);
    const float2 x0 = va ? *reinterpret_cast<const float2*>(qa + d) : z;
    const float2 x1 = vb ? *reinterpret_cast<const float2*>(qb + d) : z;
    const float2 x2 = va ? *reinterpret_cast<const float2*>(qa + d + 8) : z;
    const float2 x3 = vb ? *reinterpret_cast<const float2*>(qb + d + 8) : z;
    tm_split(x0.x, x0.y, qh[ks][0], ql[ks][0]);
    tm_split(x1.x, x1.y, qh[ks][1], ql[ks][1]);
    tm_split(x2.x, x2.y, qh[ks][2], ql[ks][2]);
    tm_split(x3.x, x3.y, qh[ks][3], ql[ks][3]);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  const int mi = lane >> 3;
  int st = 0;
  for (int b0 = p0; b0 < p1; b0 += bs, st ^= 1) {
    if (b0 + bs < p1 && !(b0 == p0 && pre1)) load_block(b0 + bs, st ^ 1);
    cp_async_commit();
    cp_async_wait1();
    __syncwarp();
    const __half* kd = ksm + st * DM_KB * BA_LD;
    const __half* vd = vsm + st * DM_KB * BA_LD;
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4(kd + (16 * np + ((mi >> 1) << 3) + (lane & 7)) * BA_LD + 16 * ks + ((mi & 1) << 3), r0, r1, r2, r3);
        mma16816(s[2 * np], ql[ks], r0, r1);
        mma16816(s[2 * np], qh[ks], r0, r1);
        mma16816(s[2 * np + 1], ql[ks], r2, r3);
        mma16816(s[2 * np + 1], qh[ks], r2, r3);
      }
    }
    float bmA = -INFINITY, bmB = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tk = b0 + 8 * i + 2 * t4 + (e & 1);
        const float a = tk < p1 && slot_attended(tk, tbase, tm0, tm1) ? __fmul_rn(s[i][e], P.scale) : -INFINITY;
        s[i][e] = a;
        if (e < 2) bmA = fmaxf(bmA, a); else bmB = fmaxf(bmB, a);
      }
    }
    bmA = fmaxf(bmA, __shfl_xor_sync(0xffffffffu, bmA, 1));
    bmA = fmaxf(bmA, __shfl_xor_sync(0xffffffffu, bmA, 2));
    bmB = fmaxf(bmB, __shfl_xor_sync(0xffffffffu, bmB, 1));
    bmB = fmaxf(bmB, __shfl_xor_sync(0xffffffffu, bmB, 2));
    const float nmA = fmaxf(mA, bmA), nmB = fmaxf(mB, bmB);
    const float uA = nmA == -INFINITY ? 0.f : nmA, uB = nmB == -INFINITY ? 0.f : nmB;
    const float fA = expf(__fsub_rn(mA, uA)), fB = expf(__fsub_rn(mB, uB));
    mA = nmA;
    mB = nmB;
    float sA = 0.f, sB = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = expf(__fsub_rn(s[i][e], e < 2 ? uA : uB));
        s[i][e] = pe;
        if (e < 2) sA = __fadd_rn(sA, pe); else sB = __fadd_rn(sB, pe);
      }
    }
    sA = __fadd_rn(sA, __shfl_xor_sync(0xffffffffu, sA, 1));
    sA = __fadd_rn(sA, __shfl_xor_sync(0xffffffffu, sA, 2));
    sB = __fadd_rn(sB, __shfl_xor_sync(0xffffffffu, sB, 1));
    sB = __fadd_rn(sB, __shfl_xor_sync(0xffffffffu, sB, 2));
    lA = fmaf(lA, fA, sA);
    lB = fmaf(lB, fB, sB);
#pragma unroll
    for (int i = 0; i < 16; ++i) { o[i][0] *= fA; o[i][1] *= fA; o[i][2] *= fB; o[i][3] *= fB; }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t ah[4], al[4];
      tm_split(s[2 * j][0], s[2 * j][1], ah[0], al[0]);
      tm_split(s[2 * j][2], s[2 * j][3], ah[1], al[1]);
      tm_split(s[2 * j + 1][0], s[2 * j + 1][1], ah[2], al[2]);
      tm_split(s[2 * j + 1][2], s[2 * j + 1][3], ah[3], al[3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vd + (16 * j + ((mi & 1) << 3) + (lane & 7)) * BA_LD + 16 * dp + ((mi >> 1) << 3), r0, r1, r2, r3);
        mma16816(o[2 * dp], al, r0, r1);
        mma16816(o[2 * dp], ah, r0, r1);
        mma16816(o[2 * dp + 1], al, r2, r3);
        mma16816(o[2 * dp + 1], ah, r2, r3);
      }
    }
    __syncwarp();   // the stage is refilled by the next iteration's prefetch
  }
}

template <int G>
__global__ void __launch_bounds__(32) k_dattn_mma(const __grid_constant__ DAttnParams P) {
  constexpr int HD = 128, PLD = HD + 4;
  extern __shared__ __align__(16) uint8_t dm_sm[];
  __half* ksm = reinterpret_cast<__half*>(dm_sm);   // [2][DM_KB][BA_LD]
  __half* vsm = ksm + 2 * DM_KB * BA_LD;
  const int t = blockIdx.x, kv = blockIdx.y, sp = blockIdx.z, lane = threadIdx.x, grp = lane >> 2, t4 = lane & 3;
  pdl_trigger();   // the merge may launch now; it reads the partials after its own dependency wait
  if (lane == 0) KQ_TRACE_AT(P.trace_id, 0);
  if (!P.st) pdl_wait();
  int n = (P.st ? P.st->pos : P.pos[t]) + 1;
  if (n > P.ctx || n < 1) {
    if (lane == 0 && sp == 0 && kv == 0 && P.err) atomicOr(P.err, KQ_DEV_ERR_BAD_POS);
    n = n < 1 ? 1 : P.ctx;
  }
  const int per = (n + P.nsplit - 1) / P.nsplit;
  const int p0 = min(n, sp * per), p1 = min(n, p0 + per);
  float o[16][4];
  float mA, mB, lA, lB;
  dm_warp_pass<G>(P, t, kv, n, p0, DM_KB, p1, ksm, vsm, o, mA, mB, lA, lB);
  // partial of rows 0..G-1 (row grp in elements 0-1, row grp + 8 in elements 2-3)
  const bool va = grp < G, vb = grp + 8 < G;
  float* part = P.part + (((size_t)t * P.n_kv + kv) * P.nsplit + sp) * G * PLD;
  if (va) {
    float* pr = part + (size_t)grp * PLD;
#pragma unroll
    for (int i = 0; i < 16; ++i) __stcg(reinterpret_cast<float2*>(pr + 8 * i + 2 * t4), make_float2(o[i][0], o[i][1]));
    if (t4 == 0) { __stcg(pr + HD, mA); __stcg(pr + HD + 1, lA); }
  }
  if (vb) {
    float* pr = part + (size_t)(grp + 8) * PLD;
#pragma unroll
    for (int i = 0; i < 16; ++i) __stcg(reinterpret_cast<float2*>(pr + 8 * i + 2 * t4), make_float2(o[i][2], o[i][3]));
    if (t4 == 0) { __stcg(pr + HD, mB); __stcg(pr + HD + 1, lB); }
  }
  if (lane == 0) KQ_TRACE_AT(P.trace_id, 4);
}

// grid (token, KV head, query head), DM_MERGE_THREADS threads: the split weights exp(m_s - M) and
// the denominator once per block in shared memory, then four groups of 128 threads (one per
// output column) each sum a quarter of the splits' rows and the groups' sums are added in group
// order. Every thread issues its quarter's row loads before the weights are known, so the block
// waits for one L2 round trip, not two. The result goes to the packed o-GEMM input or, for the
// decode step, to fp32.
constexpr int DM_MERGE_THREADS = 512;
constexpr int DM_PER_LANE = (DA_MAX_SPLIT + 31) / 32;   // splits weighed per lane of the first warp
template <int G>
__global__ void __launch_bounds__(DM_MERGE_THREADS) k_dattn_merge(const __grid_constant__ DAttnParams P) {
  constexpr int HD = 128, PLD = HD + 4, NQ = DM_MERGE_THREADS / HD, PER_MAX = (DA_MAX_SPLIT + NQ - 1) / NQ;
  __shared__ float s_w[DA_MAX_SPLIT];
  __shared__ float s_o[NQ][HD];
  __shared__ float s_L;
  const int t = blockIdx.x, kv = blockIdx.y, g = blockIdx.z, tid = threadIdx.x, lane = tid & 31;
  // the next kernel (the o GEMV) may become resident now and request its weights while the
  // partials finish; it reads this kernel's output only after its own dependency wait
  pdl_trigger();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 6);
  pdl_wait();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 7);
  const int ns = P.nsplit;
  const float* pb = P.part + ((size_t)t * P.n_kv + kv) * ns * G * PLD + (size_t)g * PLD;
  const int q = tid / HD, d = tid % HD, per = (ns + NQ - 1) / NQ, s0 = q * per, s1 = min(ns, s0 + per);
  float ov[PER_MAX];
#pragma unroll
  for (int j = 0; j < PER_MAX; ++j) ov[j] = s0 + j < s1 ? __ldcg(pb + (size_t)(s0 + j) * G * PLD + d) : 0.f;
  if (tid < 32) {
    // (m, l) of splits lane, lane + 32, ...: one 8-byte load each
    float2 ml[DM_PER_LANE];
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < DM_PER_LANE; ++j) {
      const int sp = lane + 32 * j;
      ml[j] = sp < ns ? __ldcg(reinterpret_cast<const float2*>(pb + (size_t)sp * G * PLD + HD)) : make_float2(-INFINITY, 0.f);
      M = fmaxf(M, ml[j].x);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
#pragma unroll
    for (int j = 0; j < DM_PER_LANE; ++j) {
      const float w = ml[j].x == -INFINITY ? 0.f : expf(__fsub_rn(ml[j].x, M));
      if (w != 0.f) L = __fmaf_rn(w, ml[j].y, L);
      if (lane + 32 * j < ns) s_w[lane + 32 * j] = w;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L = __fadd_rn(L, __shfl_xor_sync(0xffffffffu, L, off));
    if (lane == 0) s_L = L;
  }
  __syncthreads();
  float O = 0.f;
#pragma unroll
  for (int j = 0; j < PER_MAX; ++j) {
    if (s0 + j < s1) {
      const float wt = s_w[s0 + j];
      if (wt != 0.f) O = __fmaf_rn(wt, ov[j], O);
    }
  }
  s_o[q][d] = O;
  __syncthreads();
  if (q == 0) {
    float v = s_o[0][d];
#pragma unroll
    for (int k = 1; k < NQ; ++k) v = __fadd_rn(v, s_o[k][d]);
    v = __fdiv_rn(v, s_L);
    const int col = (kv * G + g) * HD + d;
    if (P.out_f) P.out_f[(size_t)t * P.n_kv * G * HD + col] = v;
    else xp_store(P.out_xp, P.Npad, t, col, v);
  }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 8);
}

// Tensor-parallel head: per-token (best value, global id) of this rank's vocabulary slice, whose
// first id is idx_off (lowest id on ties).
__global__ void __launch_bounds__(256) k_argmax_rows_vi(const float* logits, int V, int idx_off, float* out_v, int* out_i) {
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
    out_v[t] = v;
    out_i[t] = (vi == 0x7fffffff ? 0 : vi) + idx_off;
  }
}
// The best over the ranks' gathered rows [W][ld] for each of M tokens: rank order is id order,
// so a strict > keeps the lowest id on ties.
__global__ void k_pick_rows(const float* val, const int* idx, int W, int ld, int M, int* out) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= M) return;
  float v = val[t];
  int vi = idx[t];
  for (int r = 1; r < W; ++r)
    if (val[(size_t)r * ld + t] > v) { v = val[(size_t)r * ld + t]; vi = idx[(size_t)r * ld + t]; }
  out[t] = vi;
}

}  // namespace kq
