// kq_decode.cuh -- one decode token in ONE persistent kernel (sm_100a).
//
// The per-token work of kc_step (scripts/kindi_q4/kindi/kcpu4.c:303-335) is a chain of 5 phases
// per layer (qkv GEMV + rotary + K/V store, attention, o GEMV, gate/up GEMV + SwiGLU, down GEMV)
// and the output head. Launched as separate kernels, every phase pays a launch, a cold start of
// its weight stream and a tail. Here one CTA per SM runs all phases in order:
//
//  * One byte ring in shared memory carries, for every phase in turn, this CTA's weight stages
//    (whole 8-row tiles, one cp.async.bulk each) and, for attention phases, its K/V chunks.
//    Stages of any size sit back to back (a stage that would cross the end starts again at 0),
//    up to DEC_NB of them in flight, each with its own full / empty mbarrier pair.
//    One thread of a producer warpgroup issues the copies as soon as ring space frees up; the
//    warpgroup hands its registers to the 12 consumer warps (setmaxnreg). Copies depend only on
//    ring space, never on activations, so while the CTA waits at a phase boundary the ring
//    already fills with the next phase's bytes.
//  * The consumer warps run the phase: the GEMV pieces of kq_gemv.cuh (prologue, stages,
//    epilogues) or split-K attention over the ring. At the end of a phase every CTA adds one to
//    the phase's arrival counter; the next phase starts when the counter reaches the grid size
//    (a software grid barrier: bar.sync, one fence + atomic per CTA, acquire polling).
//  * All CTAs must be resident at once: the host launches the kernel cooperatively (one CTA per
//    SM), which fails instead of hanging when they cannot be. Every wait is bounded; a failure
//    sets the device error word, every other waiter sees it and unwinds, the producer drains its
//    copies in flight, and the host clears the counters before the next launch.
//  * The last CTA to finish re-arms the counters for the next token.
#pragma once
#include "kq_common.cuh"
#include "kq_gemv.cuh"
#include "kq_attn.cuh"

namespace kq {

enum { PH_GEMV = 0, PH_ATTN = 1 };
constexpr int DEC_RPG = 4;
constexpr int DEC_CONSUMERS = KQ_GEMV_MAX_CONSUMERS;        // 12 consumer warps (3 warpgroups)
constexpr int DEC_THREADS = DEC_CONSUMERS + 128;            // + the producer warpgroup
// Register split (setmaxnreg): the block launches with 512 x 128 registers; the producer
// warpgroup gives back down to 40 so that the consumers can take 152:
// 384 * 152 + 128 * 40 = 63488 <= 512 * 128 = 65536. Everything the producer runs after its
// setmaxnreg.dec is inlined, so ptxas fits it in 40 registers.
constexpr int DEC_REGS_CONSUMER = 152, DEC_REGS_PRODUCER = 40;
static_assert(DEC_CONSUMERS * DEC_REGS_CONSUMER + 128 * DEC_REGS_PRODUCER <= DEC_THREADS * 128, "register split");
constexpr int DEC_CWARPS = DEC_CONSUMERS / 32;
constexpr int DEC_BAR_ATTN = 12, DEC_BAR_PHASE = 13;        // named barriers (ids 1..8: GEMV rows)
constexpr uint32_t DEC_GRID_WAIT_LIMIT = 1u << 24;          // polls (~seconds) before giving up
constexpr int DEC_NB = 16;                                  // stages in flight (mbarrier pairs)
constexpr int DEC_NDESC = 4;                                // phase descriptors cached in shared memory

struct alignas(16) PhaseDesc {
  int kind;
  GemvParams g;          // PH_GEMV (its nslots / stage_bytes are unused: the kernel's ring is)
  AttnSplitParams a;     // PH_ATTN
};

struct DecodeParams {
  const PhaseDesc* ph;
  int nph;               // phases to run (the head phase is left out by a feed)
  int ring_bytes;        // byte ring at shared offset 0
  int work_off, desc_off, bars_off;   // shared-memory carve-up (desc: DEC_NDESC PhaseDesc)
  int* bar;              // [nph_total + 1] phase arrival counters; the last one is the exit ticket
  int nbar;
  DecodeState* st;
  int* err;
};

__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t cnt) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(cnt) : "memory");
}

// Bounded wait that also gives up as soon as an error has been flagged anywhere.
__device__ __forceinline__ bool mbar_wait_abort(uint64_t* bar, uint32_t parity, int* err, int bit) {
  for (uint32_t it = 0; it < KQ_WAIT_LIMIT; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 1023) == 1023 && *(volatile int*)err) return false;
  }
  atomicOr(err, bit);
  return false;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The attention work item of this CTA: kv head and its position range [t_begin, t_end).
struct AttnItem {
  int kv, sp, t_begin, t_end, nch;
  bool valid;
};
__device__ __forceinline__ AttnItem attn_item(const AttnSplitParams& S, int pos) {
  AttnItem it;
  const int b = blockIdx.x;
  it.valid = b < S.a.n_kv * S.nsplit;
  it.kv = it.valid ? b / S.nsplit : 0;
  it.sp = it.valid ? b % S.nsplit : 0;
  const int n = pos + 1;
  const int per = ((n + S.nsplit - 1) / S.nsplit + 15) & ~15;
  it.t_begin = min(n, it.sp * per);
  it.t_end = min(n, it.t_begin + per);
  it.nch = it.valid ? (it.t_end - it.t_begin + ATT_P - 1) / ATT_P : 0;
  return it;
}

// Attention scratch inside the work region (floats).
template <int G>
struct AttnScratch {
  static constexpr int sc = 0;                         // [G][ATT_P] scores / probabilities
  static constexpr int m = sc + G * ATT_P;             // [G] running max
  static constexpr int l = m + G;                      // [G] running sum
  static constexpr int f = l + G;                      // [G] rescale factor of the last chunk
  static constexpr int L = f + G;                      // [G] merged denominator
  static constexpr int last = L + G;                   // 1 int: this CTA merges
  static constexpr int red = (last + 1 + 3) & ~3;      // [8][G][128] warp partials (16-byte aligned)
  static constexpr int pm = red + 8 * G * 128;         // [ATT_SPLITS_MAX][G] partial maxima
  static constexpr int pl = pm + ATT_SPLITS_MAX * G;   // [ATT_SPLITS_MAX][G] partial sums
  static constexpr int w = pl + ATT_SPLITS_MAX * G;    // [ATT_SPLITS_MAX][G] merge weights
  static constexpr int total = w + ATT_SPLITS_MAX * G;
};

// The producer (one thread of the producer warpgroup) walks the phases' stages of this CTA in ring
// order and allocates each one in the byte ring. Positions are monotonic byte counters; stage i
// occupies [h_i, h_i + bytes_i) taken modulo the ring size, and is issued once every stage that
// ended at or before h_i + bytes_i - ring_bytes has been released (and at most DEC_NB stages are
// in flight, one mbarrier pair each).
struct RingBook {      // written by the producer before it arrives on the stage's full barrier
  int off[DEC_NB];
  int end[DEC_NB];
};

// Request phase q's descriptor into cache entry q % DEC_NDESC (one bulk copy).
__device__ __forceinline__ void fetch_desc(const DecodeParams& D, PhaseDesc* cache, uint64_t* cbar, int q) {
  if (q >= D.nph) return;
  uint64_t* bar = &cbar[q % DEC_NDESC];
  mbar_arrive_expect_tx(bar, (uint32_t)sizeof(PhaseDesc));
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(&cache[q % DEC_NDESC])), "l"(&D.ph[q]), "r"((uint32_t)sizeof(PhaseDesc)),
               "r"(smem_u32(bar)) : "memory");
}

// Descriptor of phase q in the shared cache once its copy has landed (the consumers request
// phase q + DEC_NDESC when they finish phase q). Bounded wait.
__device__ __forceinline__ const PhaseDesc* wait_desc(const DecodeParams& D, const PhaseDesc* cache, uint64_t* cbar, int q) {
  if (!mbar_wait_abort(&cbar[q % DEC_NDESC], (uint32_t)(q / DEC_NDESC) & 1, D.err, KQ_DEV_ERR_WAIT_EMPTY)) return nullptr;
  return &cache[q % DEC_NDESC];
}

// K/V rows of attention chunk c that come by bulk copy: those below `pos` (row `pos` is written by
// this token's qkv phase and read from global memory).
__device__ __forceinline__ int attn_chunk_rows(const AttnItem& itm, int c, int pos) {
  const int c0 = itm.t_begin + c * ATT_P, cnt = min(ATT_P, itm.t_end - c0);
  return max(0, min(c0 + cnt, pos) - c0);
}

// Returns the number of stages issued (all of them unless a wait gave up or an error was flagged).
__device__ __forceinline__ int dec_producer(const DecodeParams& D, RingBook& B, uint8_t* ring, uint64_t* full,
                                        uint64_t* empty, const PhaseDesc* cache, uint64_t* cbar, int apos,
                                        volatile int* s_fail) {
  const uint64_t pol = l2_evict_first_policy();
  int issued = 0, cons = 0, h = 0, T = 0;
  for (int p = 0; p < D.nph; ++p) {
    const PhaseDesc* php = wait_desc(D, cache, cbar, p);
    if (!php || *s_fail) return issued;
    const PhaseDesc& ph = *php;
    int n0 = 0, n1 = 0;
    AttnItem itm;
    if (ph.kind == PH_GEMV) {
      cta_stage_range(ph.g, n0, n1);
    } else {
      itm = attn_item(ph.a, apos);
      n1 = itm.nch;
    }
    int segi = 0;
    for (int s = n0; s < n1;) {
      const uint8_t* src;
      const __half* vsrc = nullptr;
      uint32_t bytes;
      int cnt = 1;
      if (ph.kind == PH_GEMV) {
        bytes = gemv_stage_src(ph.g, s, segi, &src);   // also moves segi to s's segment
        cnt = gemv_group(ph.g, s, n1, segi);
        for (int j = 1; j < cnt; ++j) {
          const uint8_t* s2;
          bytes += gemv_stage_src(ph.g, s + j, segi, &s2);   // contiguous tiles of one segment
        }
      } else {
        const int c0 = itm.t_begin + s * ATT_P;
        bytes = (uint32_t)attn_chunk_rows(itm, s, apos) * 128 * 2;
        src = reinterpret_cast<const uint8_t*>(ph.a.a.kc + ((size_t)itm.kv * ph.a.a.ctx + c0) * 128);
        vsrc = ph.a.a.vc + ((size_t)itm.kv * ph.a.a.ctx + c0) * 128;
      }
      const int total = (int)(vsrc ? 2 * bytes : bytes);
      const int r = h % D.ring_bytes;
      if (r + total > D.ring_bytes) h += D.ring_bytes - r;   // does not fit before the end: wrap
      // wait for the oldest stages to be released until this one fits
      while (issued - cons >= DEC_NB || h + total - T > D.ring_bytes) {
        if (!mbar_wait_abort(&empty[cons % DEC_NB], (uint32_t)(cons / DEC_NB) & 1, D.err, KQ_DEV_ERR_WAIT_EMPTY) || *s_fail)
          return issued;
        T = B.end[cons % DEC_NB];
        ++cons;
      }
      if (s == n0) KQ_TRACE_AT(p, 8);
      const int slot = issued % DEC_NB;
      const int off = h % D.ring_bytes;
      B.off[slot] = off;
      B.end[slot] = h + total;
      h += total;
      mbar_arrive_expect_tx(&full[slot], (uint32_t)total);
      if (bytes) {
        bulk_g2s(ring + off, src, bytes, &full[slot], pol);
        if (vsrc) bulk_g2s(ring + off + bytes, vsrc, bytes, &full[slot], pol);
      }
      ++issued;
      s += cnt;
    }
    KQ_TRACE_AT(p, 9);
  }
  return issued;
}

// Consumers: wait for stage `ri` to land; its byte offset in the ring, or -1 on timeout / error.
__device__ __forceinline__ int wait_stage(const DecodeParams& D, const RingBook& B, uint64_t* full, int ri) {
  const int slot = ri % DEC_NB;
  if (!mbar_wait_abort(&full[slot], (uint32_t)(ri / DEC_NB) & 1, D.err, KQ_DEV_ERR_WAIT_FULL)) return -1;
  return *(const volatile int*)&B.off[slot];
}

// Consumers of one attention phase (threads 0..255 compute; the other consumer warps wait at
// the phase barrier). Chunk c of the item arrives in ring stage `ri`; its rows below `pos` came
// by bulk copy, row `pos` (written by this token's qkv phase) is read from global memory.
template <int G>
__device__ void dec_attn(const AttnSplitParams& S, float* wk, const DecodeParams& D, const RingBook& B,
                         const uint8_t* ring, uint64_t* full, uint64_t* empty, int ri, int pos, bool& fail) {
  constexpr int HD = 128;
  using AS = AttnScratch<G>;
  const AttnParams& P = S.a;
  const AttnItem itm = attn_item(S, pos);
  if (!itm.valid) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, hl = lane & 15, half = lane >> 4;
  float* s_sc = wk + AS::sc;
  float* s_m = wk + AS::m;
  float* s_l = wk + AS::l;
  float* s_f = wk + AS::f;
  const __half* kglob = P.kc + ((size_t)itm.kv * P.ctx) * HD;
  const __half* vglob = P.vc + ((size_t)itm.kv * P.ctx) * HD;
  const int tbase = P.st->tree_base;
  const unsigned long long tm0 = P.st->mask[0], tm1 = P.st->mask[1];
  float qv[G][8];
#pragma unroll
  for (int gh = 0; gh < G; ++gh) {
    const float4* src = reinterpret_cast<const float4*>(P.q + (size_t)(itm.kv * G + gh) * HD + 8 * hl);
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
  named_bar(DEC_BAR_ATTN, ATT_THREADS);
  for (int c = 0; c < itm.nch; ++c, ++ri) {
    const int c0 = itm.t_begin + c * ATT_P, cnt = min(ATT_P, itm.t_end - c0);
    const int slot = ri % DEC_NB;
    int off = 0;
    if (!fail) {
      off = wait_stage(D, B, full, ri);
      if (off < 0) { fail = true; off = 0; }
    }
    if (tid == 0 && c == 0) KQ_TRACE_AT(S.a.trace_id, 4);
    const __half* kch = reinterpret_cast<const __half*>(ring + off);
    const __half* vch = kch + (size_t)attn_chunk_rows(itm, c, pos) * HD;
    // ---- scores
#pragma unroll
    for (int it = 0; it < ATT_IT; ++it) {
      const int tl = it * 16 + warp * 2 + half;
      const int t = c0 + tl;
      float kf[8];
      const uint4 kr = (t == pos) ? __ldcg(reinterpret_cast<const uint4*>(kglob + (size_t)pos * HD + 8 * hl))
                                  : *reinterpret_cast<const uint4*>(kch + (size_t)tl * HD + 8 * hl);
      h8_to_f(kr, kf);
#pragma unroll
      for (int gh = 0; gh < G; ++gh) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a = __fmaf_rn(kf[i], qv[gh][i], a);
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
        if (tl < cnt && hl == 0)
          s_sc[gh * ATT_P + tl] = slot_attended(t, tbase, tm0, tm1) ? __fmul_rn(a, P.scale) : -INFINITY;
      }
    }
    named_bar(DEC_BAR_ATTN, ATT_THREADS);
    if (warp < G) {
      float m = -FLT_MAX;
      for (int t = lane; t < cnt; t += 32) m = fmaxf(m, s_sc[warp * ATT_P + t]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      const float m_old = s_m[warp], m_new = fmaxf(m_old, m);
      float l = 0.f;
      for (int t = lane; t < cnt; t += 32) {
        const float e = expf(__fsub_rn(s_sc[warp * ATT_P + t], m_new));
        s_sc[warp * ATT_P + t] = e;
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
    named_bar(DEC_BAR_ATTN, ATT_THREADS);
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      const float f = s_f[gh];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[gh][i] = __fmul_rn(acc[gh][i], f);
    }
#pragma unroll
    for (int it = 0; it < ATT_IT; ++it) {
      const int tl = it * 16 + warp * 2 + half;
      const int t = c0 + tl;
      if (tl < cnt) {
        float vf[8];
        const uint4 vr = (t == pos) ? __ldcg(reinterpret_cast<const uint4*>(vglob + (size_t)pos * HD + 8 * hl))
                                    : *reinterpret_cast<const uint4*>(vch + (size_t)tl * HD + 8 * hl);
        h8_to_f(vr, vf);
#pragma unroll
        for (int gh = 0; gh < G; ++gh) {
          const float p = s_sc[gh * ATT_P + tl];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[gh][i] = __fmaf_rn(p, vf[i], acc[gh][i]);
        }
      }
    }
    named_bar(DEC_BAR_ATTN, ATT_THREADS);   // the slot and the scores are free again
    if (tid == 0) {
      mbar_arrive_cnt(&empty[slot], DEC_CWARPS);
    }
  }
  // ---- this CTA's partial (m, l, o) to global scratch
  if (tid == 0) KQ_TRACE_AT(S.a.trace_id, 5);
  float* s_red = wk + AS::red;
#pragma unroll
  for (int gh = 0; gh < G; ++gh)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[gh][i] += __shfl_xor_sync(0xffffffffu, acc[gh][i], 16);
  if (half == 0) {
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      float4* dst = reinterpret_cast<float4*>(&s_red[(warp * G + gh) * HD + 8 * hl]);
      dst[0] = make_float4(acc[gh][0], acc[gh][1], acc[gh][2], acc[gh][3]);
      dst[1] = make_float4(acc[gh][4], acc[gh][5], acc[gh][6], acc[gh][7]);
    }
  }
  named_bar(DEC_BAR_ATTN, ATT_THREADS);
  float* part = S.part + ((size_t)itm.kv * S.nsplit + itm.sp) * G * HD;
  for (int e = tid; e < G * HD; e += ATT_THREADS) {
    float o = 0.f;
#pragma unroll
    for (int r = 0; r < ATT_THREADS / 32; ++r) o += s_red[r * G * HD + e];
    __stcg(part + e, o);
  }
  if (tid < G) {
    float* ml = S.part_ml + (((size_t)itm.kv * S.nsplit + itm.sp) * G + tid) * 2;
    __stcg(ml, s_m[tid]);
    __stcg(ml + 1, s_l[tid]);
  }
  int* s_last = reinterpret_cast<int*>(wk + AS::last);
  __threadfence();
  named_bar(DEC_BAR_ATTN, ATT_THREADS);
  if (tid == 0) *s_last = (atomicAdd(&S.ticket[itm.kv], 1) == S.nsplit - 1);
  named_bar(DEC_BAR_ATTN, ATT_THREADS);
  if (!*s_last) return;
  __threadfence();
  // ---- the last CTA of the head merges the splits in split order
  float* s_pm = wk + AS::pm;
  float* s_pl = wk + AS::pl;
  float* s_w = wk + AS::w;
  float* s_L = wk + AS::L;
  const size_t mlb = (size_t)itm.kv * S.nsplit * G * 2;
  for (int e = tid; e < S.nsplit * G; e += ATT_THREADS) {
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(&S.part_ml[mlb + (size_t)e * 2]));
    s_pm[e] = ml.x;
    s_pl[e] = ml.y;
  }
  named_bar(DEC_BAR_ATTN, ATT_THREADS);
  if (tid < G) {
    float M = -FLT_MAX;
    for (int s2 = 0; s2 < S.nsplit; ++s2) M = fmaxf(M, s_pm[s2 * G + tid]);
    float Lsum = 0.f;
    for (int s2 = 0; s2 < S.nsplit; ++s2) {
      const float w = expf(__fsub_rn(s_pm[s2 * G + tid], M));
      s_w[s2 * G + tid] = w;
      Lsum = __fmaf_rn(w, s_pl[s2 * G + tid], Lsum);
    }
    s_L[tid] = Lsum;
  }
  named_bar(DEC_BAR_ATTN, ATT_THREADS);
  const float* pb = S.part + (size_t)itm.kv * S.nsplit * G * HD;
  for (int e = tid; e < G * HD; e += ATT_THREADS) {
    const int gh = e / HD;
    float v[ATT_SPLITS_MAX];
#pragma unroll
    for (int j = 0; j < ATT_SPLITS_MAX; ++j) v[j] = j < S.nsplit ? __ldcg(pb + (size_t)j * G * HD + e) : 0.f;
    float O = 0.f;
#pragma unroll
    for (int j = 0; j < ATT_SPLITS_MAX; ++j)
      if (j < S.nsplit) O = __fmaf_rn(s_w[j * G + gh], v[j], O);
    P.out[(size_t)itm.kv * G * HD + e] = __fdiv_rn(O, s_L[gh]);
  }
  if (tid == 0) S.ticket[itm.kv] = 0;
  if (tid == 0) KQ_TRACE_AT(S.a.trace_id, 6);
}

template <int G>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_decode(const __grid_constant__ DecodeParams D) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* work = smem + D.work_off;
  PhaseDesc* cache = reinterpret_cast<PhaseDesc*>(smem + D.desc_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + D.bars_off);
  uint64_t* empty = full + DEC_NB;
  uint64_t* cbar = empty + DEC_NB;
  __shared__ int s_pos, s_rpos, s_fail;
  __shared__ RingBook book;
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < DEC_NB; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], DEC_CWARPS); }
    for (int i = 0; i < DEC_NDESC; ++i) mbar_init(&cbar[i], 1);
    fence_mbar_init();
    for (int q = 0; q < DEC_NDESC; ++q) fetch_desc(D, cache, cbar, q);
    s_pos = D.st->pos;
    s_rpos = D.st->rpos;
    s_fail = 0;
  }
  __syncthreads();
  const int pos = s_pos;
  const bool pos_ok = pos >= 0 && pos < D.ph[0].g.ctx;
  const int apos = pos_ok ? pos : 0;   // positions used for attention ranges (the host validates)
  if (!pos_ok && tid == 0 && blockIdx.x == 0) atomicOr(D.err, KQ_DEV_ERR_BAD_POS);
  if (tid >= DEC_CONSUMERS) {
    // ---------------------------------------------------------------- producer warpgroup
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(DEC_REGS_PRODUCER));
    if (tid != DEC_CONSUMERS) return;
    const int issued = dec_producer(D, book, ring, full, empty, cache, cbar, apos, &s_fail);
    if (*(volatile int*)D.err) {
      // failure path only: let every copy in flight land before the CTA exits
      for (int j = max(0, issued - DEC_NB); j < issued; ++j)
        if (!mbar_wait(&full[j % DEC_NB], (uint32_t)(j / DEC_NB) & 1, D.err, KQ_DEV_ERR_DRAIN)) break;
    }
    return;
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(DEC_REGS_CONSUMER));
  int ri = 0;
  bool fail = false;
  for (int p = 0; p < D.nph; ++p) {
    // wait until every CTA has finished phase p - 1 (the producer keeps filling the ring)
    if (p > 0) {
      if (tid == 0) {
        bool ok = false;
        for (uint32_t it = 0; it < DEC_GRID_WAIT_LIMIT; ++it) {
          if (ld_acquire(&D.bar[p - 1]) >= (int)gridDim.x) { ok = true; break; }
          if ((it & 63) == 63 && *(volatile int*)D.err) break;
          __nanosleep(20);
        }
        if (!ok) {
          atomicOr(D.err, KQ_DEV_ERR_GRID);
          s_fail = 1;
        }
      }
      named_bar(DEC_BAR_PHASE, DEC_CONSUMERS);
      if (*(volatile int*)&s_fail) { fail = true; break; }
    }
    if (tid == 0) KQ_TRACE_AT(p, 0);
    // this phase's descriptor (requested DEC_NDESC phases ago)
    if (!fail && !mbar_wait_abort(&cbar[p % DEC_NDESC], (uint32_t)(p / DEC_NDESC) & 1, D.err, KQ_DEV_ERR_WAIT_FULL))
      fail = true;
    const PhaseDesc* desc = &cache[p % DEC_NDESC];
    if (desc->kind == PH_GEMV) {
      const GemvParams& P = desc->g;
      const int lane_thr = P.LPR * P.NRG, nthr_c = lane_thr * P.nlanes;
      int n0, n1;
      cta_stage_range(P, n0, n1);
      if (tid < nthr_c) {
        const GemvSmem L = gemv_smem_layout(0, 0, P.LPR, P.NRG * P.nlanes, DEC_RPG, nthr_c);
        gemv_load_rope_at(P, work, L, (s_rpos >= 0 && s_rpos < P.ctx) ? s_rpos : 0);
        // two items per thread at a time keeps the prologue's registers within the kernel's
        // budget; a norm needs every item at once and is limited to two (the host checks). One
        // call site: two inlined copies of the prologue cost far more registers than one.
        {
          const int nblk = P.xmode == XS_PLAIN ? KQ_MAX_ITEMS / 2 : 1;
#pragma unroll 1
          for (int ib = 0; ib < nblk; ++ib) gemv_prologue<2>(P, work, L, nthr_c, 2 * ib, ib == nblk - 1);
        }
        if (tid == 0) KQ_TRACE_AT(p, 1);
        GemvThread T;
        gemv_thread_init(P, work, L, pos, T);
        gemv_load_xs(P, work, L, T);
        const int lw = lane_thr >> 5;                       // warps in this lane
        const bool leader = tid % lane_thr == 0;
        int segi = 0, k = 0, e = 0;
#ifdef KQ_TRACE
        unsigned long long wait_ns = 0;
#endif
        // ring entries of this CTA's stages, dealt round-robin to the lanes
        for (int s = n0; s < n1; ++e) {
          while (s >= P.seg[segi].stage0 + P.seg[segi].nstage) ++segi;
          const int cnt = gemv_group(P, s, n1, segi);
          if (e % P.nlanes == T.lane) {
            const int rs = ri + e, slot = rs % DEC_NB;
            // after a failure the loop still runs (on whatever the ring holds) so that every
            // thread keeps taking the same barriers; the phase barrier below then ends the kernel
            int off = 0;
#ifdef KQ_TRACE
            unsigned long long tw0;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(tw0));
#endif
            if (tid == 0 && s == n0) KQ_TRACE_AT(p, 10);
            if (!fail) {
              off = wait_stage(D, book, full, rs);
              if (off < 0) { fail = true; off = 0; }
            }
#ifdef KQ_TRACE
            if (tid == 0) {
              unsigned long long tw1;
              asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(tw1));
              wait_ns += tw1 - tw0;
            }
#endif
            if (tid == 0 && s == n0) KQ_TRACE_AT(p, 4);
            const int type = P.seg[segi].w.type;
            const size_t sb = (size_t)(P.TR >> 3) * tile_bytes(type, P.G);   // bytes of a full stage
            for (int j = 0; j < cnt; ++j, ++k) {
              uint64_t* rel = j == cnt - 1 ? &empty[slot] : nullptr;   // release after the last loads
              if (type == Q4K)
                gemv_stage<TM_Q4K, DEC_RPG>(P, T, s + j, segi, ring + off + j * sb, rel, k & 1);
              else
                gemv_stage<TM_Q6K, DEC_RPG>(P, T, s + j, segi, ring + off + j * sb, rel, k & 1);
            }
            if (leader && lw < DEC_CWARPS) mbar_arrive_cnt(&empty[slot], DEC_CWARPS - lw);
          }
          s += cnt;
        }
        if (tid == 0) KQ_TRACE_AT(p, 2);
#ifdef KQ_TRACE
        if (tid == 0 && p < KQ_TRACE_LAUNCHES && blockIdx.x < KQ_TRACE_CTAS) g_kq_trace[p][blockIdx.x][5] = wait_ns;
#endif
        if (!fail && P.seg[0].epi == EPI_ARGMAX) gemv_argmax_tail<DEC_RPG>(P, work, L, T, nthr_c);
      }
      ri += gemv_group_count(P, n0, n1);   // every thread keeps the ring index in step, idle ones too
    } else {
      const AttnSplitParams& S = desc->a;
      const AttnItem itm = attn_item(S, apos);
      if (tid < ATT_THREADS)
        dec_attn<G>(S, reinterpret_cast<float*>(work), D, book, ring, full, empty, ri, apos, fail);
      ri += itm.nch;
      if (tid == 0) KQ_TRACE_AT(p, 2);
    }
    // arrive: every warp of this CTA is done with phase p (its global writes issued)
    if (fail) *(volatile int*)&s_fail = 1;
    named_bar(DEC_BAR_PHASE, DEC_CONSUMERS);
    if (*(volatile int*)&s_fail) { fail = true; break; }
    if (tid == 0) {
      KQ_TRACE_AT(p, 3);
      __threadfence();
      atomicAdd(&D.bar[p], 1);
      fetch_desc(D, cache, cbar, p + DEC_NDESC);   // this phase's cache entry is free again
    }
  }
  if (fail) {
    if (tid == 0) atomicOr(D.err, KQ_DEV_ERR_GRID);   // the producer drains; the host clears the counters
    return;
  }
  // the last CTA out re-arms the counters for the next token
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&D.bar[D.nbar - 1], 1) == (int)gridDim.x - 1) {
      for (int i = 0; i < D.nbar; ++i) D.bar[i] = 0;
      __threadfence();
    }
  }
}

}  // namespace kq
