// kq_attn.cuh -- GQA decode attention over the fp16 K/V cache (one query token).
//
// Replaces k_attn_s4w -> k_softmax_rows -> k_attn_v4p -> k_attn_comb
// (scripts/kindi_q4/kindi/kindi.cu:523-632) and the CPU restatement kcpu4.c:244-282, without
// the sigmoid output gate and with score scale 1/sqrt(head_dim).
//
// Cache layout: [n_kv][ctx][head_dim] fp16 per layer (head-major, so one split streams one
// contiguous run). Grid (n_kv, nsplit): CTA (kv, s) owns positions [s*P, s*P + P) of the
// kv-th head for its G = n_heads / n_kv query heads. Every K and V row of the split is loaded
// into registers up front -- before griddepcontrol.wait for all positions but the current one,
// which the preceding QKV kernel writes -- so the split costs one memory round trip. Scores are
// fp32 dots of the fp16 K rows with the query times the scale; the split keeps (max, sum of exp)
// and the unnormalised P.V. The last CTA of each kv head (atomic ticket) merges the splits in
// split order with the exp(m_s - M) rescaling, so the result does not depend on arrival order.
#pragma once
#include "kq_common.cuh"
#include "kq_gemv.cuh"

namespace kq {

constexpr int ATT_P = 64;              // positions per split
constexpr int ATT_THREADS = 256;       // 8 warps; a half-warp per position, 8 dims per lane
constexpr int ATT_IT = ATT_P / 16;     // positions per half-warp
constexpr int ATT_MAX_SPLITS = 1024;   // the merge keeps G x nsplit weights in shared memory

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
  int trace_id;
};

__device__ __forceinline__ void h8_to_f(const uint4 r, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) { const float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
}

template <int G>
__global__ void __launch_bounds__(ATT_THREADS) k_attn_decode(const __grid_constant__ AttnParams P) {
  constexpr int HD = 128;
  __shared__ __align__(16) float s_sc[G][ATT_P];
  __shared__ float s_m[G], s_l[G], s_L[G];
  __shared__ __align__(16) float s_red[ATT_THREADS / 32][G][HD];   // per-warp partial o (float4 stores)
  __shared__ int s_last;
  const int kv = blockIdx.x, sp = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, hl = lane & 15, half = lane >> 4;
  pdl_trigger();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 0);
  // The step's position is written before the step starts (host or the previous step's head),
  // so it can be read before waiting on the QKV kernel; only row `pos` itself is produced there.
  int pos = P.st->pos;
  const bool pos_ok = pos >= 0 && pos < P.ctx;
  if (!pos_ok) pos = pos < 0 ? 0 : P.ctx - 1;
  const int n = pos + 1;
  const int nact = (n + ATT_P - 1) / ATT_P;
  const int t0 = sp * ATT_P, cnt = sp < nact ? min(ATT_P, n - t0) : 0;
  const __half* kbase = P.kc + ((size_t)kv * P.ctx) * HD;
  const __half* vbase = P.vc + ((size_t)kv * P.ctx) * HD;
  // ---- prefetch the K and V rows of every position before `pos`
  uint4 kr[ATT_IT], vr[ATT_IT];
#pragma unroll
  for (int it = 0; it < ATT_IT; ++it) {
    const int tl = it * 16 + warp * 2 + half;
    kr[it] = make_uint4(0, 0, 0, 0);
    vr[it] = make_uint4(0, 0, 0, 0);
    if (tl < cnt && t0 + tl < pos) {
      kr[it] = __ldcs(reinterpret_cast<const uint4*>(kbase + (size_t)(t0 + tl) * HD + 8 * hl));
      vr[it] = __ldcs(reinterpret_cast<const uint4*>(vbase + (size_t)(t0 + tl) * HD + 8 * hl));
    }
  }
  pdl_wait();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 1);
  if (!pos_ok && tid == 0 && sp == 0 && kv == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_POS);
  if (sp >= nact) return;
  // ---- the current position's row (written by the QKV kernel) and the query
#pragma unroll
  for (int it = 0; it < ATT_IT; ++it) {
    const int tl = it * 16 + warp * 2 + half;
    if (tl < cnt && t0 + tl == pos) {
      kr[it] = __ldcg(reinterpret_cast<const uint4*>(kbase + (size_t)pos * HD + 8 * hl));
      vr[it] = __ldcg(reinterpret_cast<const uint4*>(vbase + (size_t)pos * HD + 8 * hl));
    }
  }
  float qv[G][8];
#pragma unroll
  for (int gh = 0; gh < G; ++gh) {
    const float4* src = reinterpret_cast<const float4*>(P.q + (size_t)(kv * G + gh) * HD + 8 * hl);
    const float4 a = __ldcg(src), b = __ldcg(src + 1);
    qv[gh][0] = a.x; qv[gh][1] = a.y; qv[gh][2] = a.z; qv[gh][3] = a.w;
    qv[gh][4] = b.x; qv[gh][5] = b.y; qv[gh][6] = b.z; qv[gh][7] = b.w;
  }
  // ---- scores
#pragma unroll
  for (int it = 0; it < ATT_IT; ++it) {
    const int tl = it * 16 + warp * 2 + half;
    float kf[8];
    h8_to_f(kr[it], kf);
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) a = __fmaf_rn(kf[i], qv[gh][i], a);
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
      if (tl < cnt && hl == 0) s_sc[gh][tl] = __fmul_rn(a, P.scale);
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
  // ---- P.V partial
  float acc[G][8];
#pragma unroll
  for (int gh = 0; gh < G; ++gh)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[gh][i] = 0.f;
#pragma unroll
  for (int it = 0; it < ATT_IT; ++it) {
    const int tl = it * 16 + warp * 2 + half;
    if (tl < cnt) {
      float vf[8];
      h8_to_f(vr[it], vf);
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
#pragma unroll
    for (int r = 0; r < ATT_THREADS / 32; ++r) o += s_red[r][gh][d];
    __stcg(part + e, o);
  }
  if (tid < G) {
    float* ml = P.part_ml + (((size_t)kv * P.nsplit + sp) * G + tid) * 2;
    __stcg(ml, s_m[tid]);
    __stcg(ml + 1, s_l[tid]);
  }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 2);
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(&P.ticket[kv], 1) == nact - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- merge the splits in order: per head M = max m_s, weights w_s = e^(m_s - M) (shared
  // memory), L = sum w_s l_s; then O = sum w_s o_s with the split loop unrolled so that its
  // loads are in flight together. Lane-strided sums end in a fixed shuffle tree: deterministic.
  float* s_w = &s_red[0][0][0];          // reused: [G][nact] weights (nact <= ATT_MAX_SPLITS)
  const size_t mlb = (size_t)kv * P.nsplit * G * 2;
  if (warp < G) {
    const int gh = warp;
    float M = -FLT_MAX;
    for (int s2 = lane; s2 < nact; s2 += 32) M = fmaxf(M, __ldcg(&P.part_ml[mlb + ((size_t)s2 * G + gh) * 2]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
    for (int s2 = lane; s2 < nact; s2 += 32) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(&P.part_ml[mlb + ((size_t)s2 * G + gh) * 2]));
      const float w = expf(__fsub_rn(ml.x, M));
      s_w[gh * nact + s2] = w;
      L = __fmaf_rn(w, ml.y, L);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    if (lane == 0) s_L[gh] = L;
  }
  __syncthreads();
  const float* pb = P.part + (size_t)kv * P.nsplit * G * HD;
  for (int e = tid; e < G * HD; e += ATT_THREADS) {
    const int gh = e / HD;
    float O = 0.f;
    for (int s0 = 0; s0 < nact; s0 += 16) {
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = s0 + j < nact ? __ldcg(pb + (size_t)(s0 + j) * G * HD + e) : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (s0 + j < nact) O = __fmaf_rn(s_w[gh * nact + s0 + j], v[j], O);
    }
    P.out[(size_t)kv * G * HD + e] = __fdiv_rn(O, s_L[gh]);
  }
  if (tid == 0) P.ticket[kv] = 0;
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 3);
}

}  // namespace kq
