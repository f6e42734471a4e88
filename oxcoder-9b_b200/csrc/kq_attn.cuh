// kq_attn.cuh -- GQA decode attention over the fp16 K/V cache (one query token).
//
// Replaces k_attn_s4w -> k_softmax_rows -> k_attn_v4p -> k_attn_comb
// (scripts/kindi_q4/kindi/kindi.cu:523-632) and the CPU restatement kcpu4.c:244-282, without
// the sigmoid output gate and with score scale 1/sqrt(head_dim).
//
// Cache layout: [n_kv][ctx][head_dim] fp16 per layer (head-major, so one split streams one
// contiguous run). Grid (n_kv, nsplit): CTA (kv, s) owns positions [s*P, s*P + P) of the
// kv-th head for its G = n_heads / n_kv query heads: scores (fp32 dot of fp16 K with the query,
// times the scale), softmax statistics (max, sum of exp) and the unnormalised P.V partial. The
// last CTA of each kv head (atomic ticket) merges the partials in split order with the usual
// exp(m_s - M) rescaling, so the result does not depend on the arrival order.
#pragma once
#include "kq_common.cuh"
#include "kq_gemv.cuh"

namespace kq {

constexpr int ATT_P = 128;      // positions per split
constexpr int ATT_THREADS = 256;

struct AttnParams {
  const float* q;        // [n_heads][hd] (rotated)
  const __half* kc;      // [n_kv][ctx][hd]
  const __half* vc;
  float* part;           // [n_kv][nsplit][G][hd]
  float* part_ml;        // [n_kv][nsplit][G][2]
  int* ticket;           // [n_kv]
  float* out;            // [n_heads][hd]
  DecodeState* st;
  int n_kv, ctx, nsplit;
  float scale;
  int* err;
};

template <int G>
__global__ void __launch_bounds__(ATT_THREADS) k_attn_decode(const __grid_constant__ AttnParams P) {
  constexpr int HD = 128;
  __shared__ __align__(16) float s_sc[G][ATT_P];
  __shared__ float s_m[G], s_l[G];
  __shared__ __align__(16) float s_red[ATT_THREADS / 32][G][HD];   // per-warp partial o (float4 stores)
  __shared__ int s_last;
  const int kv = blockIdx.x, sp = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, hl = lane & 15, half = lane >> 4;
  pdl_trigger();
  pdl_wait();
  int pos = P.st->pos;
  if (pos < 0 || pos >= P.ctx) {
    if (tid == 0 && sp == 0 && kv == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_POS);
    pos = pos < 0 ? 0 : P.ctx - 1;
  }
  const int n = pos + 1;
  const int nact = (n + ATT_P - 1) / ATT_P;
  if (sp >= nact) return;
  const int t0 = sp * ATT_P, cnt = min(ATT_P, n - t0);
  const __half* kbase = P.kc + ((size_t)kv * P.ctx) * HD;
  const __half* vbase = P.vc + ((size_t)kv * P.ctx) * HD;

  float qv[G][8];
#pragma unroll
  for (int gh = 0; gh < G; ++gh) {
    const float4* src = reinterpret_cast<const float4*>(P.q + (size_t)(kv * G + gh) * HD + 8 * hl);
    const float4 a = src[0], b = src[1];
    qv[gh][0] = a.x; qv[gh][1] = a.y; qv[gh][2] = a.z; qv[gh][3] = a.w;
    qv[gh][4] = b.x; qv[gh][5] = b.y; qv[gh][6] = b.z; qv[gh][7] = b.w;
  }
  // ---- scores: half-warp per position, 8 dims per lane
  const int iters = (cnt + 15) / 16;
  for (int it = 0; it < iters; ++it) {
    const int tl = it * 16 + warp * 2 + half;
    const bool ok = tl < cnt;
    uint4 kr = make_uint4(0, 0, 0, 0);
    if (ok) kr = *reinterpret_cast<const uint4*>(kbase + (size_t)(t0 + tl) * HD + 8 * hl);
    const __half2* kh = reinterpret_cast<const __half2*>(&kr);
    float kf[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 f = __half22float2(kh[i]); kf[2 * i] = f.x; kf[2 * i + 1] = f.y; }
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) a = __fmaf_rn(kf[i], qv[gh][i], a);
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
      if (ok && hl == 0) s_sc[gh][tl] = __fmul_rn(a, P.scale);
    }
  }
  __syncthreads();
  // ---- softmax statistics: warp gh handles head gh
  if (warp < G) {
    float m = -FLT_MAX;
    for (int t = lane; t < cnt; t += 32) m = fmaxf(m, s_sc[warp][t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float l = 0.f;
    for (int t = lane; t < cnt; t += 32) {
      const float e = expf(__fsub_rn(s_sc[warp][t], m));
      s_sc[warp][t] = e;
      l += e;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) { s_m[warp] = m; s_l[warp] = l; }
  }
  __syncthreads();
  // ---- P.V partial: same lane layout
  float acc[G][8];
#pragma unroll
  for (int gh = 0; gh < G; ++gh)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[gh][i] = 0.f;
  for (int it = 0; it < iters; ++it) {
    const int tl = it * 16 + warp * 2 + half;
    if (tl < cnt) {
      const uint4 vr = *reinterpret_cast<const uint4*>(vbase + (size_t)(t0 + tl) * HD + 8 * hl);
      const __half2* vh = reinterpret_cast<const __half2*>(&vr);
      float vf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) { const float2 f = __half22float2(vh[i]); vf[2 * i] = f.x; vf[2 * i + 1] = f.y; }
#pragma unroll
      for (int gh = 0; gh < G; ++gh) {
        const float p = s_sc[gh][tl];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[gh][i] = __fmaf_rn(p, vf[i], acc[gh][i]);
      }
    }
  }
  // the two half-warps hold the same dims for different positions: add them, then per warp
#pragma unroll
  for (int gh = 0; gh < G; ++gh)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[gh][i] += __shfl_xor_sync(0xffffffffu, acc[gh][i], 16);
  if (half == 0) {
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      float4* dst = reinterpret_cast<float4*>(&s_red[warp][gh][8 * hl]);
      dst[0] = make_float4(acc[gh][0], acc[gh][1], acc[gh][2], acc[gh][3]);
      dst[1] = make_float4(acc[gh][4], acc[gh][5], acc[gh][6], acc[gh][7]);
    }
  }
  __syncthreads();
  float* part = P.part + ((size_t)kv * P.nsplit + sp) * G * HD;
  for (int e = tid; e < G * HD; e += ATT_THREADS) {
    const int gh = e / HD, d = e % HD;
    float o = 0.f;
    for (int r = 0; r < ATT_THREADS / 32; ++r) o += s_red[r][gh][d];
    part[e] = o;
  }
  if (tid < G) {
    float* ml = P.part_ml + (((size_t)kv * P.nsplit + sp) * G + tid) * 2;
    ml[0] = s_m[tid];
    ml[1] = s_l[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(&P.ticket[kv], 1) == nact - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- merge the splits in order
  for (int e = tid; e < G * HD; e += ATT_THREADS) {
    const int gh = e / HD;
    float M = -FLT_MAX;
    for (int s = 0; s < nact; ++s) M = fmaxf(M, *(volatile float*)&P.part_ml[(((size_t)kv * P.nsplit + s) * G + gh) * 2]);
    float L = 0.f, O = 0.f;
    for (int s = 0; s < nact; ++s) {
      const size_t b = ((size_t)kv * P.nsplit + s) * G;
      const float ms = *(volatile float*)&P.part_ml[(b + gh) * 2];
      const float ls = *(volatile float*)&P.part_ml[(b + gh) * 2 + 1];
      const float f = expf(__fsub_rn(ms, M));
      L = __fmaf_rn(f, ls, L);
      O = __fmaf_rn(f, *(volatile float*)&P.part[b * HD + e], O);
    }
    P.out[(size_t)kv * G * HD + e] = __fdiv_rn(O, L);
  }
  if (tid == 0) P.ticket[kv] = 0;
}

}  // namespace kq
