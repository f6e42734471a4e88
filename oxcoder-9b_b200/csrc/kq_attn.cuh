// kq_attn.cuh -- GQA decode attention over the fp16 K/V cache (one query token).
//
// Replaces k_attn_s4w -> k_softmax_rows -> k_attn_v4p -> k_attn_comb
// (scripts/kindi_q4/kindi/kindi.cu:523-632) and the CPU restatement kcpu4.c:244-282, without
// the sigmoid output gate and with score scale 1/sqrt(head_dim).
//
// Cache layout: [n_kv][ctx][head_dim] fp16 per layer (head-major, so a CTA streams one
// contiguous run). Scores are fp32 dots of the fp16 K rows with the query times the scale.
#pragma once
#include "kq_common.cuh"
#include "kq_gemv.cuh"

namespace kq {

constexpr int ATT_P = 64;              // positions per chunk
constexpr int ATT_THREADS = 256;       // 8 warps; a half-warp per position, 8 dims per lane
constexpr int ATT_IT = ATT_P / 16;     // positions per half-warp per chunk
constexpr int ATT_MAX_CTX = 65536;

struct AttnParams {
  const float* q;        // [n_heads][hd] (rotated)
  const __half* kc;      // [n_kv][ctx][hd]
  const __half* vc;
  float* out;            // [n_heads][hd]
  DecodeState* st;
  int n_kv, ctx;
  float scale;
  int* err;
  int trace_id;
};

__device__ __forceinline__ void h8_to_f(const uint4 r, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) { const float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
}

// ------------------------------------------------------------------------------ split form
// Grid (n_kv, nsplit). CTA (kv, sp) owns the contiguous positions [sp*per, (sp+1)*per) of head kv,
// per = ceil(n / nsplit) rounded up to 16. Its K and V rows stream through a shared-memory ring
// of ATT_SLOTS chunks of ATT_P rows (one 16 KB bulk copy per chunk and tensor; chunks that do
// not hold row `pos` are requested before griddepcontrol.wait, the QKV kernel writes that row).
// Online softmax per head over the chunks; the CTA's (m, l, o) goes to global scratch and the
// last CTA of the head (atomic ticket) merges the nsplit partials in split order.
constexpr int ATT_SLOTS = 4;
constexpr int ATT_SPLITS_MAX = 32;

struct AttnSplitParams {
  AttnParams a;
  float* part;      // [n_kv][nsplit][G][hd]
  float* part_ml;   // [n_kv][nsplit][G][2]
  int* ticket;      // [n_kv]
  int nsplit;
};

template <int G>
__global__ void __launch_bounds__(ATT_THREADS, 1) k_attn_split(const __grid_constant__ AttnSplitParams S) {
  constexpr int HD = 128;
  const AttnParams& P = S.a;
  extern __shared__ __align__(128) uint8_t smem[];
  __half* ring = reinterpret_cast<__half*>(smem);                 // [ATT_SLOTS][2][ATT_P][HD]
  __shared__ __align__(8) uint64_t full[ATT_SLOTS];
  __shared__ __align__(16) float s_sc[G][ATT_P];
  __shared__ float s_m[G], s_l[G], s_f[G], s_L[G];
  __shared__ __align__(16) float s_red[ATT_THREADS / 32][G][HD];
  __shared__ int s_last;
  const int kv = blockIdx.x, sp = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, hl = lane & 15, half = lane >> 4;
  pdl_trigger();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 0);
  int pos = P.st->pos;
  const bool pos_ok = pos >= 0 && pos < P.ctx;
  if (!pos_ok) pos = pos < 0 ? 0 : P.ctx - 1;
  const int tbase = P.st->tree_base;
  const unsigned long long tm0 = P.st->mask[0], tm1 = P.st->mask[1];
  const int n = pos + 1;
  const int per = ((n + S.nsplit - 1) / S.nsplit + 15) & ~15;
  const int t_begin = min(n, sp * per), t_end = min(n, t_begin + per);
  const int nch = (t_end - t_begin + ATT_P - 1) / ATT_P;
  const __half* kbase = P.kc + ((size_t)kv * P.ctx) * HD;
  const __half* vbase = P.vc + ((size_t)kv * P.ctx) * HD;
  if (tid == 0) {
    for (int i = 0; i < ATT_SLOTS; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // chunk c: rows [t_begin + c*ATT_P, ...); the copy rounds its row count up to 8 (16-byte sizes)
  auto issue = [&](int c) {
    const int c0 = t_begin + c * ATT_P, rows = min(ATT_P, t_end - c0);
    const int rr = min((rows + 7) & ~7, P.ctx - c0);   // never past the cache's end
    const uint32_t bytes = (uint32_t)rr * HD * 2;
    uint64_t* bar = &full[c % ATT_SLOTS];
    __half* dst = ring + (size_t)(c % ATT_SLOTS) * 2 * ATT_P * HD;
    mbar_arrive_expect_tx(bar, 2 * bytes);
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(kbase + (size_t)c0 * HD), "r"(bytes), "r"(smem_u32(bar)) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst + ATT_P * HD)), "l"(vbase + (size_t)c0 * HD), "r"(bytes), "r"(smem_u32(bar)) : "memory");
  };
  // chunks that end before `pos` do not depend on the QKV kernel: request them now
  int issued = 0;
  if (tid == 0)
    while (issued < nch && issued < ATT_SLOTS && t_begin + (issued + 1) * ATT_P <= pos) issue(issued++);
  pdl_wait();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 1);
  if (!pos_ok && tid == 0 && sp == 0 && kv == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_POS);
  if (tid == 0)
    while (issued < nch && issued < ATT_SLOTS) issue(issued++);
  float qv[G][8];
#pragma unroll
  for (int gh = 0; gh < G; ++gh) {
    const float4* src = reinterpret_cast<const float4*>(P.q + (size_t)(kv * G + gh) * HD + 8 * hl);
    const float4 a = __ldcg(src), b = __ldcg(src + 1);
    qv[gh][0] = a.x; qv[gh][1] = a.y; qv[gh][2] = a.z; qv[gh][3] = a.w;
    qv[gh][4] = b.x; qv[gh][5] = b.y; qv[gh][6] = b.z; qv[gh][7] = b.w;
  }
  if (tid < G) { s_m[tid] = -FLT_MAX; s_l[tid] = 0.f; }
  float acc[G][8];
#pragma unroll
  for (int gh = 0; gh < G; ++gh)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[gh][i] = 0.f;
  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    const int c0 = t_begin + c * ATT_P, cnt = min(ATT_P, t_end - c0);
    if (!mbar_wait(&full[c % ATT_SLOTS], (uint32_t)(c / ATT_SLOTS) & 1, P.err, KQ_DEV_ERR_WAIT_FULL)) { ok = false; }
    const __half* kch = ring + (size_t)(c % ATT_SLOTS) * 2 * ATT_P * HD;
    const __half* vch = kch + ATT_P * HD;
    // ---- scores
#pragma unroll
    for (int it = 0; it < ATT_IT; ++it) {
      const int tl = it * 16 + warp * 2 + half;
      float kf[8];
      h8_to_f(*reinterpret_cast<const uint4*>(kch + (size_t)tl * HD + 8 * hl), kf);
#pragma unroll
      for (int gh = 0; gh < G; ++gh) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a = __fmaf_rn(kf[i], qv[gh][i], a);
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
        if (tl < cnt && hl == 0)
          s_sc[gh][tl] = slot_attended(c0 + tl, tbase, tm0, tm1) ? __fmul_rn(a, P.scale) : -INFINITY;
      }
    }
    __syncthreads();
    if (warp < G) {
      float m = -FLT_MAX;
      for (int t = lane; t < cnt; t += 32) m = fmaxf(m, s_sc[warp][t]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      const float m_old = s_m[warp], m_new = fmaxf(m_old, m);
      float l = 0.f;
      for (int t = lane; t < cnt; t += 32) {
        const float e = expf(__fsub_rn(s_sc[warp][t], m_new));
        s_sc[warp][t] = e;
        l += e;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) {
        const float f = expf(__fsub_rn(m_old, m_new));
        s_f[warp] = f;
        s_l[warp] = __fmaf_rn(s_l[warp], f, l);
        s_m[warp] = m_new;
      }
    }
    __syncthreads();
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      const float f = s_f[gh];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[gh][i] = __fmul_rn(acc[gh][i], f);
    }
#pragma unroll
    for (int it = 0; it < ATT_IT; ++it) {
      const int tl = it * 16 + warp * 2 + half;
      if (tl < cnt) {
        float vf[8];
        h8_to_f(*reinterpret_cast<const uint4*>(vch + (size_t)tl * HD + 8 * hl), vf);
#pragma unroll
        for (int gh = 0; gh < G; ++gh) {
          const float p = s_sc[gh][tl];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[gh][i] = __fmaf_rn(p, vf[i], acc[gh][i]);
        }
      }
    }
    __syncthreads();   // the slot and s_sc are free again
    if (tid == 0 && ok && issued < nch) issue(issued++);
  }
  // ---- this CTA's partial
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
  float* part = S.part + ((size_t)kv * S.nsplit + sp) * G * HD;
  for (int e = tid; e < G * HD; e += ATT_THREADS) {
    const int gh = e / HD, d = e % HD;
    float o = 0.f;
#pragma unroll
    for (int r = 0; r < ATT_THREADS / 32; ++r) o += s_red[r][gh][d];
    __stcg(part + e, o);
  }
  if (tid < G) {
    float* ml = S.part_ml + (((size_t)kv * S.nsplit + sp) * G + tid) * 2;
    __stcg(ml, s_m[tid]);
    __stcg(ml + 1, s_l[tid]);
  }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 2);
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(&S.ticket[kv], 1) == S.nsplit - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- merge in split order (empty splits carry m = -FLT_MAX, l = 0, o = 0)
  __shared__ float s_w[ATT_SPLITS_MAX][G];
  const size_t mlb = (size_t)kv * S.nsplit * G * 2;
  if (tid < G) {
    float M = -FLT_MAX;
    for (int s2 = 0; s2 < S.nsplit; ++s2) M = fmaxf(M, __ldcg(&S.part_ml[mlb + ((size_t)s2 * G + tid) * 2]));
    float L = 0.f;
    for (int s2 = 0; s2 < S.nsplit; ++s2) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(&S.part_ml[mlb + ((size_t)s2 * G + tid) * 2]));
      const float w = expf(__fsub_rn(ml.x, M));
      s_w[s2][tid] = w;
      L = __fmaf_rn(w, ml.y, L);
    }
    s_L[tid] = L;
  }
  __syncthreads();
  const float* pb = S.part + (size_t)kv * S.nsplit * G * HD;
  for (int e = tid; e < G * HD; e += ATT_THREADS) {
    const int gh = e / HD;
    float v[ATT_SPLITS_MAX];
#pragma unroll
    for (int j = 0; j < ATT_SPLITS_MAX; ++j) v[j] = j < S.nsplit ? __ldcg(pb + (size_t)j * G * HD + e) : 0.f;
    float O = 0.f;
#pragma unroll
    for (int j = 0; j < ATT_SPLITS_MAX; ++j)
      if (j < S.nsplit) O = __fmaf_rn(s_w[j][gh], v[j], O);
    P.out[(size_t)kv * G * HD + e] = __fdiv_rn(O, s_L[gh]);
  }
  if (tid == 0) S.ticket[kv] = 0;
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 3);
}

// ------------------------------------------------------------------------------ cluster form
// One cluster of CL CTAs per kv head (CL * n_kv CTAs in total). CTA `rank` of the
// cluster owns the contiguous positions [rank*per, (rank+1)*per), per = ceil(n / CL), and
// streams them in chunks of ATT_P positions with every K/V row of a chunk loaded up front
// (double-buffered in registers; the first chunk is requested before griddepcontrol.wait except
// for row `pos`). Softmax statistics are kept online per head (running max, rescaled sums). At
// the end each CTA leaves (m, l, o) in its shared memory; rank 0 reads the cluster's partials
// over distributed shared memory in rank order and writes the merged output. No global
// scratch, no atomics; two cluster barriers, which every CTA of the cluster executes.
constexpr int ATT_CL_MAX = 16;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ float dsmem_ld(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}

template <int G>
__device__ __forceinline__ void attn_load_chunk(const __half* kbase, const __half* vbase, int c0, int c1, int pos,
                                                bool skip_pos, int warp, int half, int hl, uint4 (&kr)[ATT_IT],
                                                uint4 (&vr)[ATT_IT]) {
  constexpr int HD = 128;
#pragma unroll
  for (int it = 0; it < ATT_IT; ++it) {
    const int t = c0 + it * 16 + warp * 2 + half;
    kr[it] = make_uint4(0, 0, 0, 0);
    vr[it] = make_uint4(0, 0, 0, 0);
    if (t < c1 && !(skip_pos && t == pos)) {
      kr[it] = __ldcs(reinterpret_cast<const uint4*>(kbase + (size_t)t * HD + 8 * hl));
      vr[it] = __ldcs(reinterpret_cast<const uint4*>(vbase + (size_t)t * HD + 8 * hl));
    }
  }
}

template <int G, int CL>
__global__ void __launch_bounds__(ATT_THREADS, 1) k_attn_cluster(const __grid_constant__ AttnParams P) {
  constexpr int HD = 128;
  __shared__ __align__(16) float s_sc[G][ATT_P];
  __shared__ float s_m[G], s_l[G], s_f[G];
  __shared__ __align__(16) float s_red[ATT_THREADS / 32][G][HD];
  __shared__ __align__(16) float s_o[G][HD];      // this CTA's partial (read by rank 0 via DSMEM)
  __shared__ float s_pm[G], s_pl[G];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, hl = lane & 15, half = lane >> 4;
  const int rank = (int)cluster_ctarank(), kv = blockIdx.x / CL;
  pdl_trigger();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 0);
  int pos = P.st->pos;
  const bool pos_ok = pos >= 0 && pos < P.ctx;
  if (!pos_ok) pos = pos < 0 ? 0 : P.ctx - 1;
  const int tbase = P.st->tree_base;
  const unsigned long long tm0 = P.st->mask[0], tm1 = P.st->mask[1];
  const int n = pos + 1;
  const int per = (n + CL - 1) / CL;
  const int t_begin = min(n, rank * per), t_end = min(n, t_begin + per);
  const __half* kbase = P.kc + ((size_t)kv * P.ctx) * HD;
  const __half* vbase = P.vc + ((size_t)kv * P.ctx) * HD;
  uint4 kr[ATT_IT], vr[ATT_IT], kn[ATT_IT], vn[ATT_IT];
  // first chunk before the wait, without row `pos` (the QKV kernel is still writing it)
  attn_load_chunk<G>(kbase, vbase, t_begin, min(t_end, t_begin + ATT_P), pos, true, warp, half, hl, kr, vr);
  pdl_wait();
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 1);
  if (!pos_ok && tid == 0 && blockIdx.x == 0) atomicOr(P.err, KQ_DEV_ERR_BAD_POS);
  {
    const int c1 = min(t_end, t_begin + ATT_P);
#pragma unroll
    for (int it = 0; it < ATT_IT; ++it) {
      const int t = t_begin + it * 16 + warp * 2 + half;
      if (t < c1 && t == pos) {
        kr[it] = __ldcg(reinterpret_cast<const uint4*>(kbase + (size_t)pos * HD + 8 * hl));
        vr[it] = __ldcg(reinterpret_cast<const uint4*>(vbase + (size_t)pos * HD + 8 * hl));
      }
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
  if (tid < G) { s_m[tid] = -FLT_MAX; s_l[tid] = 0.f; }
  float acc[G][8];
#pragma unroll
  for (int gh = 0; gh < G; ++gh)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[gh][i] = 0.f;
  for (int c0 = t_begin; c0 < t_end; c0 += ATT_P) {
    const int cnt = min(ATT_P, t_end - c0);
    // next chunk's rows in flight while this one is computed
    if (c0 + ATT_P < t_end) attn_load_chunk<G>(kbase, vbase, c0 + ATT_P, min(t_end, c0 + 2 * ATT_P), pos, false, warp, half, hl, kn, vn);
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
        if (tl < cnt && hl == 0)
          s_sc[gh][tl] = slot_attended(c0 + tl, tbase, tm0, tm1) ? __fmul_rn(a, P.scale) : -INFINITY;
      }
    }
    __syncthreads();
    // ---- online softmax statistics (warp gh, head gh): new max, rescale factor, exps, sum
    if (warp < G) {
      float m = -FLT_MAX;
      for (int t = lane; t < cnt; t += 32) m = fmaxf(m, s_sc[warp][t]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      const float m_old = s_m[warp], m_new = fmaxf(m_old, m);
      float l = 0.f;
      for (int t = lane; t < cnt; t += 32) {
        const float e = expf(__fsub_rn(s_sc[warp][t], m_new));
        s_sc[warp][t] = e;
        l += e;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) {
        const float f = expf(__fsub_rn(m_old, m_new));
        s_f[warp] = f;
        s_l[warp] = __fmaf_rn(s_l[warp], f, l);
        s_m[warp] = m_new;
      }
    }
    __syncthreads();
    // ---- rescale and accumulate P.V
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      const float f = s_f[gh];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[gh][i] = __fmul_rn(acc[gh][i], f);
    }
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
    __syncthreads();   // s_sc / s_f reused by the next chunk
#pragma unroll
    for (int it = 0; it < ATT_IT; ++it) { kr[it] = kn[it]; vr[it] = vn[it]; }
  }
  // ---- this CTA's partial o into shared memory
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
  for (int e = tid; e < G * HD; e += ATT_THREADS) {
    const int gh = e / HD, d = e % HD;
    float o = 0.f;
#pragma unroll
    for (int r = 0; r < ATT_THREADS / 32; ++r) o += s_red[r][gh][d];
    s_o[gh][d] = o;
  }
  if (tid < G) { s_pm[tid] = s_m[tid]; s_pl[tid] = s_l[tid]; }
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 2);
  cluster_sync_all();
  // ---- rank 0 merges the cluster's partials in rank order
  if (rank == 0) {
    __shared__ float s_w[CL][G], s_L[G];
    if (tid < G) {
      float M = -FLT_MAX;
      for (int r = 0; r < CL; ++r) M = fmaxf(M, dsmem_ld(dsmem_addr(&s_pm[tid], (uint32_t)r)));
      float L = 0.f;
      for (int r = 0; r < CL; ++r) {
        const float w = expf(__fsub_rn(dsmem_ld(dsmem_addr(&s_pm[tid], (uint32_t)r)), M));
        s_w[r][tid] = w;
        L = __fmaf_rn(w, dsmem_ld(dsmem_addr(&s_pl[tid], (uint32_t)r)), L);
      }
      s_L[tid] = L;
    }
    __syncthreads();
    for (int e = tid; e < G * HD; e += ATT_THREADS) {
      const int gh = e / HD, d = e % HD;
      float v[CL];
#pragma unroll
      for (int r = 0; r < CL; ++r) v[r] = dsmem_ld(dsmem_addr(&s_o[gh][d], (uint32_t)r));
      float O = 0.f;
#pragma unroll
      for (int r = 0; r < CL; ++r) O = __fmaf_rn(s_w[r][gh], v[r], O);
      P.out[(size_t)kv * G * HD + e] = __fdiv_rn(O, s_L[gh]);
    }
  }
  cluster_sync_all();   // partials stay readable until rank 0 is done
  if (tid == 0) KQ_TRACE_AT(P.trace_id, 3);
}

}  // namespace kq
