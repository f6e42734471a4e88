// kq_api.cu -- host runtime and C ABI (include/kq.h) of the B200 Kindi-Q4 decode path.
//
// Replaces the reference's CuPy engine (scripts/kindi_q4/kindi/gpu4.py:50-110, engine.py:293-366):
// weights resident in HBM in the kq layout, one decode token = 32 x {QKV GEMV (+norm, rotary,
// K/V store), attention, o GEMV, gate/up GEMV (+norm, SwiGLU), down GEMV} + head GEMV (+norm,
// argmax), captured once into a CUDA graph with programmatic-dependent-launch edges and replayed
// per token. There is no CPU fallback: every entry point fails with KQ_ERR_BACKEND if CUDA does.
#include "../../include/kq.h"
#include "kq_common.cuh"
#include "kq_qformat.cuh"
#include "kq_gemv.cuh"
#include "kq_gemv_mma.cuh"
#include "kq_attn.cuh"
#include "kq_decode.cuh"
#include "kq_accept.cuh"
#include "kq_batch.cuh"
#include "kq_ngram.h"
#include "kq_tmv.cuh"
#include "kq_nccl.h"
#include "kq_pack.h"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <thread>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

using namespace kq;

#define KQ_VERSION 100

// ------------------------------------------------------------------------------ errors
static thread_local std::string g_err;
static int set_err(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
#define CU(call)                                                                                 \
  do {                                                                                           \
    cudaError_t e_ = (call);                                                                     \
    if (e_ != cudaSuccess) return set_err(KQ_ERR_BACKEND, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)
#define CUP(call)                                                                                \
  do {                                                                                           \
    cudaError_t e_ = (call);                                                                     \
    if (e_ != cudaSuccess) { set_err(KQ_ERR_BACKEND, std::string(#call) + ": " + cudaGetErrorString(e_)); return nullptr; } \
  } while (0)

// ------------------------------------------------------------------------------ kernel table
typedef void (*GemvFn)(GemvParams);
static GemvFn gemv_fn(int tm, int rpg) {
  static const GemvFn tab[3][3] = {
      {k_gemv<TM_Q4K, 1>, k_gemv<TM_Q4K, 2>, k_gemv<TM_Q4K, 4>},
      {k_gemv<TM_Q6K, 1>, k_gemv<TM_Q6K, 2>, k_gemv<TM_Q6K, 4>},
      {k_gemv<TM_MIXED, 1>, k_gemv<TM_MIXED, 2>, k_gemv<TM_MIXED, 4>}};
  return tab[tm - 1][rpg == 1 ? 0 : rpg == 2 ? 1 : 2];
}

// The tensor-core Q4_K GEMV for nw consumer warps, nb 16-row blocks per stage, C columns.
static GmFn gm_fn(int nw, int nb, int C, int ty) {
  if (ty == 1) {
    if (nw == 16) return nb == 2 ? gm_fn_for<16, 2, 1>(C) : gm_fn_for<16, 1, 1>(C);
    return nb == 2 ? gm_fn_for<12, 2, 1>(C) : gm_fn_for<12, 1, 1>(C);
  }
  if (nw == 16) return nb == 2 ? gm_fn_for<16, 2, 2>(C) : gm_fn_for<16, 1, 2>(C);
  return nb == 2 ? gm_fn_for<12, 2, 2>(C) : gm_fn_for<12, 1, 2>(C);
}

// ------------------------------------------------------------------------------ per-device context
struct DevCtx {
  bool init = false;
  int nsm = 0;
  int* err = nullptr;       // device error word for matrix-hook calls
  size_t smem_optin = 0;
  size_t tmm_budget = 0;    // dynamic shared memory of the tensor-core GEMM
  size_t tmv_smem = 0;      // dynamic shared memory available to k_tmv (0: the tensor-core GEMV is off)
};
static DevCtx g_dev[16];
static std::mutex g_dev_mu;

static int dev_init(int device) {
  if (device < 0 || device >= 16) return set_err(KQ_ERR_ARG, "device index out of range");
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DevCtx& d = g_dev[device];
  if (d.init) return KQ_OK;
  CU(cudaSetDevice(device));
  CU(cudaDeviceGetAttribute(&d.nsm, cudaDevAttrMultiProcessorCount, device));
  int optin = 0;
  CU(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  size_t static_max = 0;
  for (int tm = 1; tm <= 3; ++tm)
    for (int ri = 0; ri < 3; ++ri) {
      cudaFuncAttributes fa;
      CU(cudaFuncGetAttributes(&fa, gemv_fn(tm, 1 << ri)));
      static_max = std::max(static_max, (size_t)fa.sharedSizeBytes);
    }
  d.smem_optin = (size_t)optin - static_max;
  for (int tm = 1; tm <= 3; ++tm)
    for (int ri = 0; ri < 3; ++ri)
      CU(cudaFuncSetAttribute(gemv_fn(tm, 1 << ri), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)d.smem_optin));
  for (int nw : {12, 16})
    for (int nb : {1, 2})
      for (int c : {256, 12288})
        for (int ty : {1, 2})
          CU(cudaFuncSetAttribute(gm_fn(nw, nb, c, ty), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)d.smem_optin));
  {
    cudaFuncAttributes fa;
    CU(cudaFuncGetAttributes(&fa, k_tmm));
    d.tmm_budget = (size_t)optin - fa.sharedSizeBytes;
    CU(cudaFuncSetAttribute(k_tmm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)d.tmm_budget));
  }
  CU(cudaFuncSetAttribute(k_battn<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BA_SMEM));
  CU(cudaFuncSetAttribute(k_battn<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BA_SMEM));
  CU(cudaFuncSetAttribute(k_battn<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BA_SMEM));
  CU(cudaFuncSetAttribute(k_battn<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)BA_SMEM));
  {
    cudaFuncAttributes fa;
    CU(cudaFuncGetAttributes(&fa, k_tmv));
    const size_t budget = (size_t)optin - fa.sharedSizeBytes;
    CU(cudaFuncSetAttribute(k_tmv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)budget));
    const char* ev = std::getenv("KQ_TMV");   // opt-in while it is validated: 1 = the tensor-core GEMV
    d.tmv_smem = (ev && std::atoi(ev) == 1) ? budget : 0;
  }
  CU(cudaMalloc(&d.err, sizeof(int)));
  CU(cudaMemset(d.err, 0, sizeof(int)));
  d.init = true;
  return KQ_OK;
}

// ------------------------------------------------------------------------------ matrices
struct kq_qmat {
  int device = 0, type = 0, R = 0, C = 0, G = 0;
  uint8_t* buf = nullptr;   // R/8 tiles (kq layout)
  size_t bytes = 0;
  float* tv_part = nullptr; // split-K scratch of the tensor-core GEMV (matvec calls), lazily
  int* tv_ticket = nullptr;
  bool tvon = false;        // keep the unit-major copy of the tensor-core GEMV
  uint8_t* tvbuf = nullptr; // that copy (kq_tmv.cuh), rebuilt by every write
  QView view() const {
    QView v;
    v.base = buf; v.type = type; v.R = R; v.C = C; v.G = G; v.tv = tvbuf;
    return v;
  }
  QViewW wview() {
    QViewW v;
    v.base = buf; v.type = type; v.R = R; v.C = C; v.G = G;
    return v;
  }
};

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Shape rule of every quantised matrix: whole 8-row tiles, whole super-blocks, and at most 12288
// columns (the widest activation vector the digit-plane prologue and the packed batched-pass
// input hold). The tensor-core GEMM of the batched passes takes any such shape.
static int check_shape(int type, int R, int C) {
  if (type != KQ_Q4_K && type != KQ_Q6_K) return set_err(KQ_ERR_ARG, "tensor type must be 12 (Q4_K) or 14 (Q6_K)");
  if (R <= 0 || C <= 0 || R % 8 || C % 256)
    return set_err(KQ_ERR_ARG, "Invalid packed tensor dimensions: rows must be a positive multiple of 8 and cols of 256");
  if (C > 12288) return set_err(KQ_ERR_ARG, "unsupported column count (at most 12288)");
  return KQ_OK;
}

// Extra rule of the single-token GEMV (k_gemv, k_tmv, the persistent kernel): a row's C/64
// threads reduce by warp shuffles within a power-of-two segment of a warp (4, 8, 16 threads) or
// over whole warps (a multiple of 32), so C is 256, 512, 1024 or a multiple of 2048. A
// tensor-parallel shard whose slice breaks it (1536 or 3072 FFN columns) only runs the batched
// pass.
static int check_gemv_cols(int C) {
  const int LPR = 4 * (C / 256);
  if (!(LPR == 4 || LPR == 8 || LPR == 16 || (LPR % 32 == 0 && LPR <= 192)))
    return set_err(KQ_ERR_ARG, "the single-token GEMV needs 256, 512, 1024 or a multiple of 2048 columns up to 12288");
  return KQ_OK;
}

static kq_qmat* qmat_alloc(int type, int R, int C, int device) {
  if (check_shape(type, R, C) != KQ_OK) return nullptr;
  if (dev_init(device) != KQ_OK) return nullptr;
  CUP(cudaSetDevice(device));
  kq_qmat* a = new kq_qmat();
  a->device = device; a->type = type; a->R = R; a->C = C; a->G = C / 256;
  a->bytes = (size_t)R * a->G * block_bytes(type);
  if (cudaMalloc(&a->buf, a->bytes) != cudaSuccess) {
    delete a;
    set_err(KQ_ERR_MEMORY, "device allocation of a quantised matrix failed");
    return nullptr;
  }
  a->tvon = g_dev[device].tmv_smem > 0 && a->G <= TV_MAX_G;
  return a;
}

// The unit-major copy of the tensor-core GEMV, (re)built from the tile layout on stream s.
static int qmat_tv_build(kq_qmat* a, cudaStream_t s) {
  if (!a->tvon) return KQ_OK;
  const long long ntiles = (a->R + TV_ROWS - 1) / TV_ROWS, nthr = ntiles * a->G * TV_ROWS;
  if (!a->tvbuf) {
    const size_t ub = a->type == Q4K ? TV_UNIT_Q4 : TV_UNIT_Q6;
    if (cudaMalloc(&a->tvbuf, (size_t)ntiles * a->G * ub) != cudaSuccess) {
      a->tvon = false;   // the tile layout alone still serves every kernel
      cudaGetLastError();
      return KQ_OK;
    }
  }
  k_tv_repack<<<(unsigned)((nthr + 255) / 256), 256, 0, s>>>(a->view(), a->tvbuf);
  CU(cudaGetLastError());
  return KQ_OK;
}

static int qmat_write(kq_qmat* a, int R_src, const uint8_t* src_dev, uint64_t base, int mode, int arg, cudaStream_t s,
                      ShardMap sh = ShardMap{0, 0, 0}) {
  const long long n = (long long)R_src * a->G;
  const int thr = 128;
  if (sh.G_src == 0) sh.G_src = a->G;
  k_qmat_write<<<(unsigned)((n + thr - 1) / thr), thr, 0, s>>>(a->wview(), R_src, src_dev, base, mode, arg, sh);
  CU(cudaGetLastError());
  return qmat_tv_build(a, s);
}

// `pack`: the host bytes are in the Kindi pack's 8-row interleave instead of GGUF row-major order.
static int qmat_upload_mapped(kq_qmat* a, const void* host, size_t bytes, int R_src, int mode, int arg, cudaStream_t s,
                              bool pack = false) {
  const size_t need = (size_t)R_src * a->G * block_bytes(a->type);
  if (bytes != need) return set_err(KQ_ERR_ARG, "tensor byte count does not match its shape");
  uint8_t* tmp = nullptr;
  CU(cudaMalloc(&tmp, bytes));
  cudaError_t e = cudaMemcpyAsync(tmp, host, bytes, cudaMemcpyHostToDevice, s);
  int rc = KQ_OK;
  if (e != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, std::string("upload: ") + cudaGetErrorString(e));
  if (rc == KQ_OK) rc = qmat_write(a, R_src, tmp, 0, mode, arg, s, ShardMap{0, 0, 0, pack ? 1 : 0});
  cudaStreamSynchronize(s);
  cudaFree(tmp);
  return rc;
}

// ------------------------------------------------------------------------------ GEMV planning
struct GemvPlan {
  int TR, LPR, NRG, RPG, TM, stage_bytes, nslots, threads, grid;
  int tr4, tr6;  // k_gemv_mma: rows per stage of the Q4_K and of the Q6_K segments
  size_t smem;
  bool mma;      // k_gemv_mma instead of k_gemv
};

static const size_t KQ_SMEM_BUDGET = 220 * 1024;
static const int KQ_MAX_STEP_GEMVS = 4 * 256 + 8;   // GEMV launches of one step at most (4 a layer + head)

// Launch shape of a (fused) GEMV over segments sharing the column count C.
static int plan_gemv(int C, const int* types, int nseg, const int* seg_rows, bool pairs, int nsm, size_t optin,
                     GemvPlan& pl) {
  const int G = C / 256, LPR = 4 * G;
  int rowb = 0;
  bool has4 = false, has6 = false;
  for (int i = 0; i < nseg; ++i) {
    rowb = std::max(rowb, block_bytes(types[i]) * G);
    has4 |= types[i] == KQ_Q4_K;
    has6 |= types[i] == KQ_Q6_K;
  }
  const size_t budget = std::min(KQ_SMEM_BUDGET, optin);
  // tuning override for sweeps: KQ_GEMV_RPG (1, 2, 4) and KQ_GEMV_NRG fix the shape if valid
  const int want_rpg = std::getenv("KQ_GEMV_RPG") ? std::atoi(std::getenv("KQ_GEMV_RPG")) : 0;
  const int want_nrg = std::getenv("KQ_GEMV_NRG") ? std::atoi(std::getenv("KQ_GEMV_NRG")) : 0;
  // Candidates are scored: (a) when every CTA's share fits the ring (no stage waits for a slot
  // to be released), fewer stages per CTA: a stage of 24 rows costs
  // ~2.1 us of consumer time against ~1.5 us for 8 rows; then (b) more consumer warps and
  // (c) more rows per thread (activation reuse). Short stages for a deeper pipeline lost: the
  // config-0 GEMV takes 12.1 us with 8-row stages (>= 4 per CTA), 11.2 us with 24-row stages.
  bool found = false;
  long best = -1;
  for (int NRG = std::min(KQ_MAX_NRG, KQ_GEMV_MAX_CONSUMERS / LPR); NRG >= 1; --NRG) {
    if ((LPR * NRG) % 32) continue;
    if (8 * LPR > KQ_MAX_ITEMS * LPR * NRG) continue;   // prologue items per thread
    for (int RPG : {4, 2, 1}) {
      if (pairs && (RPG & 1)) continue;
      if (want_rpg && RPG != want_rpg) continue;
      if (want_nrg && NRG != want_nrg) continue;
      const int TR = NRG * RPG;
      if (TR % 8) continue;                              // stages are whole 8-row tiles
      const int stage_bytes = (int)align_up((size_t)TR * rowb, 128);
      const GemvSmem L0 = gemv_smem_layout(0, stage_bytes, LPR, NRG, RPG, LPR * NRG);
      const size_t fixed = L0.total + 64;
      if (fixed + 2 * ((size_t)stage_bytes + 16) > budget) continue;
      int nstages = 0;
      for (int i = 0; i < nseg; ++i) nstages += (seg_rows[i] + TR - 1) / TR;
      const int grid = std::max(1, std::min(nsm, nstages));
      int slots = (int)((budget - fixed) / (stage_bytes + 16));
      slots = std::min(8, std::max(2, slots));
      const int per_cta = (nstages + grid - 1) / grid;
      const long score = (per_cta <= slots ? (1L << 21) - 1024L * per_cta : 0) + (long)(LPR * NRG) * 8 + RPG;
      if (score <= best) continue;
      best = score;
      found = true;
      pl.TR = TR; pl.LPR = LPR; pl.NRG = NRG; pl.RPG = RPG;
      pl.TM = (has4 && has6) || std::getenv("KQ_GEMV_MIXED") ? TM_MIXED : has6 ? TM_Q6K : TM_Q4K;   // env: tuning
      pl.stage_bytes = stage_bytes;
      pl.nslots = slots;
      pl.smem = gemv_smem_layout(slots, stage_bytes, LPR, NRG, RPG, LPR * NRG).total;
      pl.threads = LPR * NRG + 32;
      pl.grid = grid;
    }
  }
  if (!found) return set_err(KQ_ERR_ARG, "no valid GEMV launch shape for this column count");
  pl.mma = false;
  return KQ_OK;
}

// Launch shape of the tensor-core GEMV (k_gemv_mma): Q4_K stages of 16 NB rows, Q6_K stages of
// nt6 8-row tiles, ring slots of the larger stage, as many as shared memory holds (at least 2).
// False when a segment is of another type, the shape does not fit, or KQ_GEMV_MMA=0 (a
// comparison switch) asks for k_gemv.
static bool plan_gemv_mma(int C, const int* types, int nseg, const int* seg_rows, int nsm, size_t optin, GemvPlan& pl) {
  const char* env = std::getenv("KQ_GEMV_MMA");
  if (env && std::atoi(env) == 0) return false;
  bool has4 = false, has6 = false;
  for (int i = 0; i < nseg; ++i) {
    if (types[i] != KQ_Q4_K && types[i] != KQ_Q6_K) return false;
    has4 |= types[i] == KQ_Q4_K;
    has6 |= types[i] == KQ_Q6_K;
  }
  // Q6_K: the tensor-core consumer wins inside a mixed launch (the decode step's q/k/v GEMV: its
  // compact code and one launch shape for both types) but issues more instructions per weight
  // than k_gemv's dp4a form, so a launch of Q6_K segments only stays on k_gemv (measured, Q6_K
  // 151936 x 4096: 100 us k_gemv, 147 us here; 4096 x 12288: 15.0 / 16.7 us). Comparison
  // switch KQ_GEMV_MMA6: 0 = never for Q6_K, 1 = always.
  const char* e6 = std::getenv("KQ_GEMV_MMA6");
  const int mma6 = e6 ? std::atoi(e6) : -1;
  if (has6 && mma6 == 0) return false;
  const int G = C / 256;
  // 16 consumer warps, Q4_K stages of two 16-row blocks (measured on config-0: 16 warps x 32 rows
  // 9.12 us, 8 x 32 9.19, 8 x 16 11.45, 16 x 16 11.73, k_gemv 11.07; a 226 MB launch: 43.0 /
  // 43.4 / 55.7 / 59.3 / 56.4 us; the decode step 2.16 / 2.20 / 2.34 / 2.36 / 2.45 ms).
  // Tuning overrides: KQ_GM_WARPS (12 or 16), KQ_GM_BLOCKS (1 or 2), KQ_GM6_TILES (1, 2 or 4).
  const int nw = std::getenv("KQ_GM_WARPS") && std::atoi(std::getenv("KQ_GM_WARPS")) == 12 ? 12 : 16;
  const int nb = std::getenv("KQ_GM_BLOCKS") && std::atoi(std::getenv("KQ_GM_BLOCKS")) == 1 ? 1 : 2;
  const int want6 = std::getenv("KQ_GM6_TILES") ? std::atoi(std::getenv("KQ_GM6_TILES")) : 0;
  if (G * 256 != C || C > 8 * GM_MAXI * 32 * nw) return false;
  const size_t budget = std::min(KQ_SMEM_BUDGET, optin);
  const size_t fixed = gm_smem_layout(0, 0, C).total + 64;
  const int tr4 = 16 * nb;
  const size_t b4 = has4 ? align_up((size_t)tr4 * 144 * G, 128) : 0;
  // Q6_K: the largest stage (up to 4 tiles) that still leaves two ring slots
  int nt6 = 0;
  size_t stage = 0;
  for (int nt : {4, 2, 1}) {
    if (!has6) { stage = b4; break; }
    if (want6 && nt != want6) continue;
    const size_t st = std::max(b4, align_up((size_t)nt * 8 * 210 * G, 128));
    if (fixed + 2 * (st + 16) <= budget) { nt6 = nt; stage = st; break; }
  }
  if (has6 && !nt6) return false;
  if (fixed + 2 * (stage + 16) > budget) return false;
  const int tr6 = 8 * nt6;
  int nstages = 0;
  for (int i = 0; i < nseg; ++i) {
    const int tr = types[i] == KQ_Q4_K ? tr4 : tr6;
    nstages += (seg_rows[i] + tr - 1) / tr;
  }
  // a Q6_K-only launch with many stages per CTA is streaming-bound: k_gemv's cheaper consumer
  // wins there; a short one (the decode step's down projection, ~3.5 stages per CTA) is bound by
  // the prologue, which is shorter here
  const int max_per_cta = std::getenv("KQ_MMA6_MAX_PER_CTA") ? std::atoi(std::getenv("KQ_MMA6_MAX_PER_CTA")) : 8;
  if (has6 && !has4 && mma6 < 0 && nstages > max_per_cta * nsm) return false;
  const int slots = std::min(8, (int)((budget - fixed) / (stage + 16)));
  pl.TR = std::max(has4 ? tr4 : 0, has6 ? tr6 : 0);
  pl.tr4 = tr4; pl.tr6 = tr6;
  pl.LPR = 4 * G; pl.NRG = nw; pl.RPG = nb; pl.TM = has6 ? 2 : 1;   // NRG, RPG, TM: warps, row blocks, types
  pl.stage_bytes = (int)stage;
  pl.nslots = slots;
  pl.smem = gm_smem_layout(slots, (int)stage, C).total;
  pl.threads = (nw + 1) * 32;
  pl.grid = std::max(1, std::min(nsm, nstages));
  pl.mma = true;
  return true;
}

struct SegSpec {
  const kq_qmat* m;
  int epi;
  float* out_f;
  __half* out_h;
};

static int fill_gemv(const SegSpec* ss, int nseg, bool pairs, int nsm, GemvParams& p, GemvPlan& pl) {
  if (nseg < 1 || nseg > KQ_MAX_SEG) return set_err(KQ_ERR_ARG, "bad segment count");
  int types[KQ_MAX_SEG], rows[KQ_MAX_SEG];
  const int C = ss[0].m->C;
  if (check_gemv_cols(C) != KQ_OK) return KQ_ERR_ARG;
  for (int i = 0; i < nseg; ++i) {
    if (ss[i].m->C != C) return set_err(KQ_ERR_ARG, "fused GEMV segments must share the column count");
    types[i] = ss[i].m->type;
    rows[i] = ss[i].m->R;
  }
  int rc = KQ_OK;
  if (!plan_gemv_mma(C, types, nseg, rows, nsm, g_dev[ss[0].m->device].smem_optin, pl) &&
      (rc = plan_gemv(C, types, nseg, rows, pairs, nsm, g_dev[ss[0].m->device].smem_optin, pl)))
    return rc;
  std::memset(&p, 0, sizeof(p));
  p.nseg = nseg;
  int st = 0;
  for (int i = 0; i < nseg; ++i) {
    p.seg[i].w = ss[i].m->view();
    p.seg[i].stage0 = st;
    const int tr = !pl.mma ? pl.TR : ss[i].m->type == KQ_Q4_K ? pl.tr4 : pl.tr6;
    p.seg[i].nstage = (ss[i].m->R + tr - 1) / tr;
    p.seg[i].tr = tr;
    p.seg[i].epi = ss[i].epi;
    p.seg[i].out_f = ss[i].out_f;
    p.seg[i].out_h = ss[i].out_h;
    st += p.seg[i].nstage;
  }
  p.nstages = st;
  p.C = C; p.G = C / 256; p.TR = pl.TR; p.LPR = pl.LPR; p.NRG = pl.NRG; p.nlanes = 1; p.tps = 1;
  p.stage_bytes = pl.stage_bytes; p.nslots = pl.nslots;
  // tuning override for sweeps: KQ_GEMV_PREFETCH stages go out before the prologue is done
  // (the tensor-core GEMV's stages are smaller: its whole ring goes out before the prologue ends)
  p.prefetch = std::getenv("KQ_GEMV_PREFETCH") ? std::max(0, std::atoi(std::getenv("KQ_GEMV_PREFETCH")))
                                               : pl.mma ? pl.nslots : KQ_PREFETCH_STAGES;
  return KQ_OK;
}

// Launch shape of a GEMV phase of the persistent decode kernel: its 384 threads form lanes of
// max(32, 2 * LPR) threads (LPR = C/64 threads per row, RPG 4 rows each); a lane consumes whole
// stages of TR = 4 * (lane threads / LPR) rows (one 8-row tile for C >= 1024) on its own, so
// stages are small and a CTA's share of a phase splits evenly.
static int fill_gemv_dec(const SegSpec* ss, int nseg, GemvParams& p, int& stage_bytes) {
  if (nseg < 1 || nseg > KQ_MAX_SEG) return set_err(KQ_ERR_ARG, "bad segment count");
  const int C = ss[0].m->C, G = C / 256, LPR = 4 * G;
  if (check_gemv_cols(C) != KQ_OK) return KQ_ERR_ARG;
  int rowb = 0;
  for (int i = 0; i < nseg; ++i) {
    if (ss[i].m->C != C) return set_err(KQ_ERR_ARG, "fused GEMV segments must share the column count");
    rowb = std::max(rowb, block_bytes(ss[i].m->type) * G);
  }
  const int lane_thr = std::max(32, 2 * LPR);
  if (lane_thr > DEC_CONSUMERS || lane_thr % 32) return set_err(KQ_ERR_ARG, "no persistent-kernel shape for this column count");
  const int nlanes = DEC_CONSUMERS / lane_thr, NRG = lane_thr / LPR;
  if (NRG * DEC_RPG % 8) return set_err(KQ_ERR_ARG, "no persistent-kernel shape for this column count");
  const int TR = NRG * DEC_RPG;
  const int nthr_c = lane_thr * nlanes;
  if (8 * LPR > KQ_MAX_ITEMS * nthr_c) return set_err(KQ_ERR_ARG, "persistent kernel: GEMV input too wide");
  std::memset(&p, 0, sizeof(p));
  p.nseg = nseg;
  int st = 0;
  for (int i = 0; i < nseg; ++i) {
    p.seg[i].w = ss[i].m->view();
    p.seg[i].stage0 = st;
    p.seg[i].nstage = (ss[i].m->R + TR - 1) / TR;
    p.seg[i].tr = TR;
    p.seg[i].epi = ss[i].epi;
    p.seg[i].out_f = ss[i].out_f;
    p.seg[i].out_h = ss[i].out_h;
    st += p.seg[i].nstage;
  }
  p.nstages = st;
  p.C = C; p.G = G; p.TR = TR; p.LPR = LPR; p.NRG = NRG; p.nlanes = nlanes;
  // ring entries of up to 3 stages on phases with many stages per CTA (fewer, larger copies);
  // single stages where a CTA has few (finer balance). An entry stays <= 81 KB.
  const int per_cta = std::max(1, st / std::max(1, g_dev[ss[0].m->device].nsm));
  const int tps_env = std::getenv("KQ_DEC_TPS") ? std::atoi(std::getenv("KQ_DEC_TPS")) : 0;   // tuning
  int tps = tps_env > 0 ? tps_env : std::min(3, std::max(1, per_cta / 8));
  while (tps > 1 && (size_t)tps * TR * rowb > 82560) --tps;
  p.tps = tps;
  stage_bytes = (int)align_up((size_t)tps * TR * rowb, 128);
  p.stage_bytes = stage_bytes;
  p.nslots = 0;
  return KQ_OK;
}

static cudaError_t launch_gemv(const GemvParams& p, const GemvPlan& pl, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.grid);
  cfg.blockDim = dim3((unsigned)pl.threads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  if (pl.mma) return cudaLaunchKernelEx(&cfg, gm_fn(pl.NRG, pl.RPG, p.C, pl.TM), p);
  return cudaLaunchKernelEx(&cfg, gemv_fn(pl.TM, pl.RPG), p);
}

template <int G, int CL>
static cudaError_t launch_attn_cl_t(const AttnParams& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.n_kv * CL));
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, k_attn_cluster<G, CL>, a);
}
template <int G>
static cudaError_t launch_attn_split_t(const AttnSplitParams& a, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.a.n_kv, (unsigned)a.nsplit);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = (size_t)ATT_SLOTS * 2 * ATT_P * 128 * 2;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_attn_split<G>, a);
}
static cudaError_t launch_attn_split(const AttnSplitParams& a, int G, cudaStream_t s, bool pdl) {
  switch (G) {
    case 1: return launch_attn_split_t<1>(a, s, pdl);
    case 2: return launch_attn_split_t<2>(a, s, pdl);
    case 4: return launch_attn_split_t<4>(a, s, pdl);
    default: return launch_attn_split_t<8>(a, s, pdl);
  }
}
static int attn_split_setup() {
  const int bytes = ATT_SLOTS * 2 * ATT_P * 128 * 2;
  CU(cudaFuncSetAttribute(k_attn_split<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  CU(cudaFuncSetAttribute(k_attn_split<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  CU(cudaFuncSetAttribute(k_attn_split<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  CU(cudaFuncSetAttribute(k_attn_split<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return KQ_OK;
}
typedef cudaError_t (*AttnClFn)(const AttnParams&, cudaStream_t, bool);
static AttnClFn attn_cl_fn(int G, int CL) {
  if (CL == 16) return G == 1 ? launch_attn_cl_t<1, 16> : G == 2 ? launch_attn_cl_t<2, 16> : G == 4 ? launch_attn_cl_t<4, 16> : launch_attn_cl_t<8, 16>;
  return G == 1 ? launch_attn_cl_t<1, 8> : G == 2 ? launch_attn_cl_t<2, 8> : G == 4 ? launch_attn_cl_t<4, 8> : launch_attn_cl_t<8, 8>;
}
template <int G, int CL>
static int attn_cl_setup() {
  if (CL > 8) CU(cudaFuncSetAttribute(k_attn_cluster<G, CL>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  return KQ_OK;
}
// Cluster size for the attention of `n_kv` heads: 16 CTAs per head when the device can keep
// n_kv such clusters resident at once, else 8.
static int attn_cluster_size(int G, int n_kv) {
  int rc = G == 1 ? attn_cl_setup<1, 16>() : G == 2 ? attn_cl_setup<2, 16>() : G == 4 ? attn_cl_setup<4, 16>() : attn_cl_setup<8, 16>();
  if (rc) return 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_kv * 16));
  cfg.blockDim = dim3(ATT_THREADS);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 16;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int nclusters = 0;
  const void* fn = G == 1 ? (const void*)k_attn_cluster<1, 16> : G == 2 ? (const void*)k_attn_cluster<2, 16>
                 : G == 4 ? (const void*)k_attn_cluster<4, 16> : (const void*)k_attn_cluster<8, 16>;
  if (const char* e = std::getenv("KQ_ATTN_CL")) return std::atoi(e) == 16 ? 16 : 8;   // tuning override
  const cudaError_t qe = cudaOccupancyMaxActiveClusters(&nclusters, fn, &cfg);
  if (std::getenv("KQ_VERBOSE")) std::fprintf(stderr, "kq: %d active 16-CTA attention clusters (%s)\n", nclusters, cudaGetErrorString(qe));
  if (qe != cudaSuccess) { cudaGetLastError(); return 8; }
  return nclusters >= n_kv ? 16 : 8;
}

// ------------------------------------------------------------------------------ model
struct LayerW {
  kq_qmat *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
  float *attn_norm = nullptr, *ffn_norm = nullptr;
  __half *kc = nullptr, *vc = nullptr;
  __half *bkc = nullptr, *bvc = nullptr;   // batched decode: [n_seq][n_kv][ctx][hd] per tensor
};

struct kq_model {
  kq_config c{};
  int device = 0, nsm = 0;
  // tensor parallelism (world 1: the whole model). Rank r holds KV heads [r nkv_l, (r+1) nkv_l)
  // and their query heads (q/k/v rows, o input columns, K/V cache), the FFN slice
  // [r ffn_l, (r+1) ffn_l) (gate/up rows, down input columns) and the vocabulary slice
  // [r vocab_l, ...) of the head; embedding and norms are whole on every rank. One NCCL
  // all-reduce of the o and the down outputs per layer, an all-gather of the head's argmax.
  int tp_rank = 0, tp_world = 1;
  int nh_l = 0, nkv_l = 0, ffn_l = 0, vocab_l = 0;
  ncclComm_t comm = nullptr;
  bool comm_dead = false;           // the communicator was aborted after a peer stopped answering
  // pinned staging of a batched pass's per-token metadata (tokens, slots, rotary positions,
  // sequences, masks): a ring whose slot is reused once the copies that read it have run, so the
  // uploads stay asynchronous (a pageable upload may wait for the stream, and a stream stuck in a
  // collective would then hold the host beyond the tensor-parallel deadline)
  struct MetaSlot {
    int tok[128], slot[128], rpos[128], seq[128];
    unsigned long long mask[256];
  };
  static constexpr int META_RING = 4;
  MetaSlot* meta = nullptr;
  cudaEvent_t meta_ev[META_RING] = {};
  int meta_i = 0, meta_cur = 0;
  int n_seq = 0;                    // sequences of the batched-decode caches (kq_batch_caches)
  int *bseq = nullptr, *bposv = nullptr;   // [MM_MAXM] per-token sequence / position of a batched step
  float* dpart = nullptr;           // batched decode attention partials
  float* tp_val = nullptr;          // [world][MM_MAXM] head argmax values of every rank
  int* tp_idx = nullptr;            // [world][MM_MAXM] their (global) ids
  cudaStream_t stream = nullptr;
  std::vector<LayerW> L;
  kq_qmat *emb = nullptr, *out = nullptr;
  float* out_norm = nullptr;
  float *cos_t = nullptr, *sin_t = nullptr;
  float *h[2] = {nullptr, nullptr}, *y = nullptr, *q = nullptr, *att = nullptr, *mbuf = nullptr, *logits = nullptr;
  float* hpart_val = nullptr;
  int* hpart_idx = nullptr;
  int* hticket = nullptr;
  DecodeState* st = nullptr;
  DecodeState* st_host = nullptr;   // pinned
  int* out_ids = nullptr;           // tokens of the device-resident loop
  int out_cap = 0;
  int* err = nullptr;
  int attn_cl = 16;                  // CTAs per kv head in the cluster attention
  int attn_mode = 0;                 // 0: split form, 1: cluster form, 2: tensor-core split form
  int dsplit = 0;                    // key splits of the tensor-core decode attention
  float* dpart1 = nullptr;          // decode-step partials of the tensor-core split form
  int* gdyn = nullptr;               // stage-claim counter pairs of the step's GEMV launches (zeroed)
  float* tv_part = nullptr;         // split-K scratch of the tensor-core GEMV (decode graph)
  int* tv_ticket = nullptr;
  int attn_nsplit = 1;
  float *apart = nullptr, *apart_ml = nullptr;
  int* aticket = nullptr;
  cudaGraphExec_t g_step = nullptr, g_feed = nullptr;
  int step_kernels = 0;             // kernel nodes of the decode-step graph
  // optional time split of the batched passes (KQ_PHASE_TIMES=1): an event before each launch
  // group, its category, and the accumulated ms per category (GEMM, attention, all-reduce, other)
  bool prof = false;
  std::vector<cudaEvent_t> pev;
  std::vector<int> pcat;
  size_t pn = 0;
  double pms[4] = {0, 0, 0, 0};
  // persistent decode kernel (k_decode): phase table, arrival counters, launch shape
  bool persist = true;
  PhaseDesc* d_phases = nullptr;
  int nph_all = 0;
  int* dec_bar = nullptr;
  DecodeParams dec{};
  size_t dec_smem = 0;
  // speculative verification (allocated on first use)
  float* vlogits = nullptr;         // [KQ_MAX_TREE][vocab] logits of the last verify pass
  int vn = 0;                       // nodes of the last verify pass
  DecodeState* vstates = nullptr;   // pinned, one per node
  float *ap = nullptr, *aq = nullptr, *ag = nullptr;   // acceptance scratch, draft logits
  int *atok = nullptr, *apar = nullptr, *apath = nullptr, *aout = nullptr, *acnt = nullptr;
  AccGridScratch* agrid = nullptr;   // the multi-CTA acceptance's exchange area
  float *auacc = nullptr, *aufin = nullptr;
  __half** caches = nullptr;        // [2 * n_layers] K/V cache pointers (compaction)
  // batched verification pass (up to MM_MAXM tokens at once)
  float *bh = nullptr, *by = nullptr, *bq = nullptr, *bpart = nullptr;
  __half *bxd = nullptr, *bxa = nullptr, *bxf = nullptr;   // packed GEMM inputs: C = dim, NH*HD, ffn
  float *bxs_n = nullptr, *bxs_f = nullptr;   // per-token range scales of bxd (norm) and bxf (SwiGLU)
  float *bxd_sum = nullptr, *bxf_sum = nullptr;   // their sub-block sums (xp_sub_sum; C % 256 == 0)
  float* bmf = nullptr;                       // [MM_MAXM][ffn_l] SwiGLU output before packing
  int *btok = nullptr, *bslot = nullptr, *brpos = nullptr, *bticket = nullptr;
  unsigned long long* bmask = nullptr;
  int b_nsplit = 0;                 // attention key splits the scratch holds
  float* tpart = nullptr;           // split-K partials of the tensor-core GEMM
  int* tticket = nullptr;
  size_t tpart_floats = 0;
  int tticket_n = 0;
  bool verify_seq = false;          // node-by-node decode steps instead of the batched pass
  std::vector<void*> allocs;
};

static_assert(MM_MAXM == 128, "the metadata staging slots hold MM_MAXM tokens");

static int model_check(kq_model* m) {
  if (!m) return set_err(KQ_ERR_ARG, "null model");
  CU(cudaSetDevice(m->device));
  return KQ_OK;
}

// Time split of the batched passes (KQ_PHASE_TIMES=1 only): prof_mark records an event before a
// launch group of category cat; prof_flush (after the stream synchronised) adds each interval
// between consecutive events to the category of its first event. The events separate the
// kernels, so programmatic launch overlap is lost while the split is on.
enum { PC_GEMM = 0, PC_ATTN = 1, PC_COMM = 2, PC_OTHER = 3, PC_END = 4 };
static void prof_mark(kq_model* m, int cat) {
  if (!m->prof) return;
  if (m->pn == m->pev.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) { m->prof = false; return; }
    m->pev.push_back(e);
    m->pcat.push_back(0);
  }
  cudaEventRecord(m->pev[m->pn], m->stream);
  m->pcat[m->pn++] = cat;
}
static void prof_flush(kq_model* m) {
  if (!m->prof) return;
  for (size_t i = 1; i < m->pn; ++i) {
    float ms = 0.f;
    if (m->pcat[i - 1] < PC_END && cudaEventElapsedTime(&ms, m->pev[i - 1], m->pev[i]) == cudaSuccess) m->pms[m->pcat[i - 1]] += ms;
  }
  m->pn = 0;
}


extern "C" {

int kq_version(void) { return KQ_VERSION; }
const char* kq_error(void) { return g_err.c_str(); }
int kq_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

void kq_config_default(kq_config* c) {
  if (!c) return;
  c->dim = 4096; c->n_layers = 32; c->n_heads = 32; c->n_kv_heads = 8; c->head_dim = 128; c->ffn = 12288;
  c->vocab = 151936; c->ctx = 4096; c->rope_theta = 1e6f; c->eps = 1e-6f;
  c->t_q = KQ_Q4_K; c->t_k = KQ_Q4_K; c->t_v = KQ_Q6_K; c->t_o = KQ_Q4_K; c->t_gate = KQ_Q4_K; c->t_up = KQ_Q4_K;
  c->t_down = KQ_Q6_K; c->t_emb = KQ_Q4_K; c->t_out = KQ_Q6_K;
  c->max_tokens = 64;
}

}  // extern "C"

// ------------------------------------------------------------------------------ bounded NCCL waits
// Every host wait on the peers of a tensor-parallel model ends by a deadline: KQ_TP_TIMEOUT_MS
// (default 60000) from the start of the wait. At the deadline the communicator is aborted
// (ncclCommAbort also ends this rank's collective kernels, so its stream drains), the model is
// marked dead for tensor-parallel work and the call returns KQ_ERR_TIMEOUT.
static double host_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}
static double tp_timeout_ms() {
  const char* v = std::getenv("KQ_TP_TIMEOUT_MS");
  const double t = v ? std::atof(v) : 60000.0;
  return t > 0 ? t : 60000.0;
}
static void tp_abort(kq_model* m) {
  if (m->comm) nccl().CommAbort(m->comm);
  m->comm = nullptr;
  m->comm_dead = true;
}
static void tp_comm_close(kq_model* m) {
  if (!m->comm) return;
  ncclResult_t st = nccl().CommFinalize(m->comm);
  const double end = host_ms() + 10000.0;
  while (st == ncclInProgress && host_ms() < end) {
    std::this_thread::sleep_for(std::chrono::microseconds(100));
    if (nccl().CommGetAsyncError(m->comm, &st) != ncclSuccess) break;
  }
  if (st == ncclSuccess) nccl().CommDestroy(m->comm);
  else nccl().CommAbort(m->comm);
  m->comm = nullptr;
}
// Completes a non-blocking NCCL call that returned r.
static int nccl_wait(kq_model* m, ncclResult_t r, const char* what) {
  const double end = host_ms() + tp_timeout_ms();
  while (r == ncclInProgress) {
    if (host_ms() > end) {
      tp_abort(m);
      return set_err(KQ_ERR_TIMEOUT, std::string(what) + ": a tensor-parallel peer did not answer in time; the communicator was aborted");
    }
    std::this_thread::yield();
    if (nccl().CommGetAsyncError(m->comm, &r) != ncclSuccess) break;
  }
  if (r != ncclSuccess) {
    const std::string msg = std::string(what) + ": " + nccl().GetErrorString(r);
    tp_abort(m);
    return set_err(KQ_ERR_BACKEND, msg);
  }
  return KQ_OK;
}
// The end of a pass: the model's stream drained, for a tensor-parallel model with the peers'
// health polled and the wait bounded.
static int tp_sync(kq_model* m) {
  if (m->tp_world == 1 || !m->comm) {
    CU(cudaStreamSynchronize(m->stream));
    return KQ_OK;
  }
  const double start = host_ms(), end = start + tp_timeout_ms();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(m->stream);
    if (q == cudaSuccess) return KQ_OK;
    if (q != cudaErrorNotReady) return set_err(KQ_ERR_BACKEND, std::string("tensor-parallel pass: ") + cudaGetErrorString(q));
    ncclResult_t st = ncclSuccess;
    nccl().CommGetAsyncError(m->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      const std::string msg = std::string("NCCL: ") + nccl().GetErrorString(st);
      tp_abort(m);
      cudaStreamSynchronize(m->stream);
      return set_err(KQ_ERR_BACKEND, msg);
    }
    const double now = host_ms();
    if (now > end) {
      tp_abort(m);
      cudaStreamSynchronize(m->stream);   // the aborted collectives return; the stream drains
      char buf[160];
      std::snprintf(buf, sizeof buf, "a tensor-parallel peer did not answer within %.0f ms; the communicator was aborted",
                    tp_timeout_ms());
      return set_err(KQ_ERR_TIMEOUT, buf);
    }
    if (now - start > 2.0) std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}
static int tp_alive(const kq_model* m) {
  if (m->comm_dead) return set_err(KQ_ERR_BACKEND, "the tensor-parallel communicator was aborted after a peer stopped answering");
  return KQ_OK;
}
// An event of the model's stream has completed; bounded like tp_sync for a tensor-parallel model.
static int tp_wait_event(kq_model* m, cudaEvent_t ev) {
  if (m->tp_world == 1 || !m->comm) {
    CU(cudaEventSynchronize(ev));
    return KQ_OK;
  }
  const double end = host_ms() + tp_timeout_ms();
  for (;;) {
    const cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return KQ_OK;
    if (q != cudaErrorNotReady) return set_err(KQ_ERR_BACKEND, std::string("tensor-parallel pass: ") + cudaGetErrorString(q));
    if (host_ms() > end) return tp_sync(m);   // aborts the communicator and reports the timeout
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}
// The next metadata slot, once the uploads that last read it have run.
static int meta_acquire(kq_model* m, kq_model::MetaSlot** out) {
  if (!m->meta) {
    CU(cudaMallocHost(&m->meta, sizeof(kq_model::MetaSlot) * kq_model::META_RING));
    for (cudaEvent_t& e : m->meta_ev) CU(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  const int i = m->meta_i++ % kq_model::META_RING;
  int rc = tp_wait_event(m, m->meta_ev[i]);
  if (rc) return rc;
  m->meta_cur = i;
  *out = &m->meta[i];
  return KQ_OK;
}
// After the uploads from the current slot are enqueued.
static int meta_release(kq_model* m) {
  CU(cudaEventRecord(m->meta_ev[m->meta_cur], m->stream));
  return KQ_OK;
}

static void model_release(kq_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream && m->comm) tp_sync(m);   // bounded: a silent peer gets the communicator aborted
  if (m->stream) cudaStreamSynchronize(m->stream);
  if (m->comm && nccl().ok) tp_comm_close(m);
  if (m->g_step) cudaGraphExecDestroy(m->g_step);
  if (m->g_feed) cudaGraphExecDestroy(m->g_feed);
  for (auto& l : m->L) {
    kq_qmat* ms[] = {l.q, l.k, l.v, l.o, l.gu, l.down};
    for (kq_qmat* a : ms)
      if (a) { cudaFree(a->buf); cudaFree(a->tvbuf); delete a; }
  }
  for (kq_qmat* a : {m->emb, m->out})
    if (a) { cudaFree(a->buf); cudaFree(a->tvbuf); delete a; }
  for (void* p : m->allocs) cudaFree(p);
  if (m->st_host) cudaFreeHost(m->st_host);
  if (m->vstates) cudaFreeHost(m->vstates);
  for (cudaEvent_t e : m->pev) cudaEventDestroy(e);
  for (cudaEvent_t e : m->meta_ev)
    if (e) cudaEventDestroy(e);
  if (m->meta) cudaFreeHost(m->meta);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

template <typename T>
static T* dalloc(kq_model* m, size_t n, bool& ok) {
  void* p = nullptr;
  if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) { ok = false; return nullptr; }
  cudaMemset(p, 0, n * sizeof(T));
  m->allocs.push_back(p);
  return reinterpret_cast<T*>(p);
}

static int validate_cfg(const kq_config& c) {
  if (c.head_dim != 128) return set_err(KQ_ERR_ARG, "head_dim must be 128");
  if (c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads) return set_err(KQ_ERR_ARG, "n_heads must be a multiple of n_kv_heads");
  const int G = c.n_heads / c.n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return set_err(KQ_ERR_ARG, "query heads per kv head must be 1, 2, 4 or 8");
  if (c.dim < 512) return set_err(KQ_ERR_ARG, "dim must be at least 512");
  if (c.n_heads * c.head_dim < 512) return set_err(KQ_ERR_ARG, "n_heads * head_dim must be at least 512");
  if (c.ctx < 1 || c.ctx > ATT_MAX_CTX) return set_err(KQ_ERR_ARG, "ctx out of range (1 .. 65536)");
  if (c.vocab <= 0 || c.vocab % 8) return set_err(KQ_ERR_ARG, "vocab must be a positive multiple of 8");
  if (c.t_gate != c.t_up) return set_err(KQ_ERR_ARG, "gate and up must share a quantisation type");
  if (c.n_layers < 1) return set_err(KQ_ERR_ARG, "n_layers must be positive");
  const int shapes[][3] = {{c.t_q, c.n_heads * c.head_dim, c.dim}, {c.t_k, c.n_kv_heads * c.head_dim, c.dim},
                           {c.t_v, c.n_kv_heads * c.head_dim, c.dim}, {c.t_o, c.dim, c.n_heads * c.head_dim},
                           {c.t_gate, 2 * c.ffn, c.dim}, {c.t_down, c.dim, c.ffn},
                           {c.t_emb, c.vocab, c.dim}, {c.t_out, c.vocab, c.dim}};
  // the whole model runs the single-token GEMV in its decode graph (tensor-parallel shards are
  // checked by qmat_alloc with the generic rule only)
  for (auto& s : shapes)
    if (check_shape(s[0], s[1], s[2]) != KQ_OK || check_gemv_cols(s[2]) != KQ_OK) return KQ_ERR_ARG;
  return KQ_OK;
}

static kq_model* model_create(const kq_config* cfg, int device, int rank, int world) {
  if (!cfg) { set_err(KQ_ERR_ARG, "null config"); return nullptr; }
  if (validate_cfg(*cfg) != KQ_OK) return nullptr;
  if (world < 1 || rank < 0 || rank >= world) { set_err(KQ_ERR_ARG, "bad tensor-parallel rank / world"); return nullptr; }
  if (world > 1 && (cfg->n_kv_heads % world || (cfg->ffn / world) % 256 || cfg->vocab % world ||
                    ((cfg->n_heads / world) * cfg->head_dim) % 256)) {
    set_err(KQ_ERR_ARG, "tensor-parallel split needs n_kv_heads, vocab divisible by world and 256-column slices");
    return nullptr;
  }
  if (dev_init(device) != KQ_OK) return nullptr;
  CUP(cudaSetDevice(device));
  kq_model* m = new kq_model();
  m->c = *cfg;
  m->device = device;
  m->nsm = g_dev[device].nsm;
  m->tp_rank = rank;
  m->tp_world = world;
  const kq_config& c = m->c;
  m->nh_l = c.n_heads / world;
  m->nkv_l = c.n_kv_heads / world;
  m->ffn_l = c.ffn / world;
  m->vocab_l = c.vocab / world;
  bool ok = true;
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) ok = false;
  const int QD = m->nh_l * c.head_dim, KD = m->nkv_l * c.head_dim;
  m->L.resize(c.n_layers);
  for (int l = 0; ok && l < c.n_layers; ++l) {
    LayerW& w = m->L[l];
    w.q = qmat_alloc(c.t_q, QD, c.dim, device);
    w.k = qmat_alloc(c.t_k, KD, c.dim, device);
    w.v = qmat_alloc(c.t_v, KD, c.dim, device);
    w.o = qmat_alloc(c.t_o, c.dim, QD, device);
    w.gu = qmat_alloc(c.t_gate, 2 * m->ffn_l, c.dim, device);
    w.down = qmat_alloc(c.t_down, c.dim, m->ffn_l, device);
    if (!w.q || !w.k || !w.v || !w.o || !w.gu || !w.down) { ok = false; break; }
    w.attn_norm = dalloc<float>(m, c.dim, ok);
    w.ffn_norm = dalloc<float>(m, c.dim, ok);
    w.kc = dalloc<__half>(m, (size_t)KD * c.ctx, ok);
    w.vc = dalloc<__half>(m, (size_t)KD * c.ctx, ok);
  }
  if (ok) {
    m->emb = qmat_alloc(c.t_emb, c.vocab, c.dim, device);
    m->out = qmat_alloc(c.t_out, m->vocab_l, c.dim, device);
    if (!m->emb || !m->out) ok = false;
    else m->emb->tvon = m->out->tvon = false;   // the embedding and the head run on k_gemv
  }
  if (ok && world > 1) {
    m->tp_val = dalloc<float>(m, (size_t)(world + 1) * MM_MAXM, ok);   // gathered rows + this rank's
    m->tp_idx = dalloc<int>(m, (size_t)(world + 1) * MM_MAXM, ok);
  }
  const int rh = c.head_dim / 2;
  if (ok) {
    m->out_norm = dalloc<float>(m, c.dim, ok);
    m->cos_t = dalloc<float>(m, (size_t)c.ctx * rh, ok);
    m->sin_t = dalloc<float>(m, (size_t)c.ctx * rh, ok);
    m->h[0] = dalloc<float>(m, c.dim, ok);
    m->h[1] = dalloc<float>(m, c.dim, ok);
    m->y = dalloc<float>(m, c.dim, ok);
    m->q = dalloc<float>(m, QD, ok);
    m->att = dalloc<float>(m, QD, ok);
    m->mbuf = dalloc<float>(m, c.ffn, ok);
    m->logits = dalloc<float>(m, c.vocab, ok);
    m->attn_cl = attn_cluster_size(c.n_heads / c.n_kv_heads, c.n_kv_heads);
    m->attn_mode = std::getenv("KQ_ATTN") ? std::atoi(std::getenv("KQ_ATTN")) : 2;   // tuning override
    if (m->attn_mode < 0 || m->attn_mode > 2) m->attn_mode = 2;
    m->dsplit = std::getenv("KQ_DSPLIT") ? std::atoi(std::getenv("KQ_DSPLIT")) : DA_MAX_SPLIT;   // tuning override
    if (m->dsplit < 1 || m->dsplit > DA_MAX_SPLIT) m->dsplit = DA_MAX_SPLIT;
    m->dpart1 = dalloc<float>(m, (size_t)c.n_kv_heads * DA_MAX_SPLIT * (c.n_heads / c.n_kv_heads) * (c.head_dim + 4), ok);
    if (!(std::getenv("KQ_GEMV_DYN") && std::atoi(std::getenv("KQ_GEMV_DYN")) == 0))
      m->gdyn = dalloc<int>(m, (size_t)2 * KQ_MAX_STEP_GEMVS, ok);
    m->persist = std::getenv("KQ_PERSIST") && std::atoi(std::getenv("KQ_PERSIST")) == 1;   // opt-in for now
    m->verify_seq = std::getenv("KQ_VERIFY_SEQ") && std::atoi(std::getenv("KQ_VERIFY_SEQ")) == 1;
    m->prof = std::getenv("KQ_PHASE_TIMES") && std::atoi(std::getenv("KQ_PHASE_TIMES")) == 1;
    m->attn_nsplit = std::min(ATT_SPLITS_MAX, std::max(1, m->nsm / c.n_kv_heads));
    m->apart = dalloc<float>(m, (size_t)c.n_kv_heads * m->attn_nsplit * (c.n_heads / c.n_kv_heads) * c.head_dim, ok);
    m->apart_ml = dalloc<float>(m, (size_t)c.n_kv_heads * m->attn_nsplit * (c.n_heads / c.n_kv_heads) * 2, ok);
    m->aticket = dalloc<int>(m, c.n_kv_heads, ok);
    m->tv_part = dalloc<float>(m, (size_t)m->nsm * 2 * TV_ROWS, ok);
    m->tv_ticket = dalloc<int>(m, (size_t)TV_MAX_TILES, ok);
    if (attn_split_setup() != KQ_OK) ok = false;
    m->hpart_val = dalloc<float>(m, 1024, ok);
    m->hpart_idx = dalloc<int>(m, 1024, ok);
    m->hticket = dalloc<int>(m, 1, ok);
    m->st = dalloc<DecodeState>(m, 1, ok);
    m->out_cap = c.ctx;
    m->out_ids = dalloc<int>(m, (size_t)m->out_cap, ok);
    m->err = dalloc<int>(m, 1, ok);
    if (cudaMallocHost(&m->st_host, sizeof(DecodeState)) != cudaSuccess) ok = false;
  }
  if (ok) {
    // RoPE tables as cpu4.py:175-178: fp64 angles, cast to f32.
    std::vector<float> ct((size_t)c.ctx * rh), stb((size_t)c.ctx * rh);
    for (int p = 0; p < c.ctx; ++p)
      for (int i = 0; i < rh; ++i) {
        const double inv = std::pow((double)c.rope_theta, -2.0 * (double)i / (double)c.head_dim);
        const double th = (double)p * inv;
        ct[(size_t)p * rh + i] = (float)std::cos(th);
        stb[(size_t)p * rh + i] = (float)std::sin(th);
      }
    if (cudaMemcpy(m->cos_t, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->sin_t, stb.data(), stb.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      ok = false;
  }
  if (!ok || cudaDeviceSynchronize() != cudaSuccess) {
    if (g_err.empty() || g_err.find("alloc") == std::string::npos) set_err(KQ_ERR_MEMORY, "model allocation failed");
    model_release(m);
    return nullptr;
  }
  return m;
}

extern "C" kq_model* kq_model_create(const kq_config* cfg, int device) { return model_create(cfg, device, 0, 1); }

extern "C" int kq_tp_unique_id(uint8_t* out128) {
  if (!out128) return set_err(KQ_ERR_ARG, "null id buffer");
  if (!nccl().ok) return set_err(KQ_ERR_BACKEND, "NCCL could not be loaded");
  ncclUniqueId id;
  const ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess) return set_err(KQ_ERR_BACKEND, std::string("ncclGetUniqueId: ") + nccl().GetErrorString(r));
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
  std::memcpy(out128, &id, 128);
  return KQ_OK;
}

// Every rank calls this with the same id (from kq_tp_unique_id on one rank); it returns once all
// `world` ranks have joined the communicator.
extern "C" kq_model* kq_model_create_tp(const kq_config* cfg, int device, int rank, int world, const uint8_t* id128) {
  if (!id128 && world > 1) { set_err(KQ_ERR_ARG, "null NCCL id"); return nullptr; }
  kq_model* m = model_create(cfg, device, rank, world);
  if (!m || world == 1) return m;
  if (!nccl().ok) { set_err(KQ_ERR_BACKEND, "NCCL could not be loaded"); model_release(m); return nullptr; }
  ncclUniqueId id;
  std::memcpy(&id, id128, 128);
  ncclConfig_t cfgc = NCCL_CONFIG_INITIALIZER;
  cfgc.blocking = 0;   // every wait on the peers is then a host poll with a deadline
  const ncclResult_t r = nccl().CommInitRankConfig(&m->comm, world, id, rank, &cfgc);
  if (r != ncclSuccess && r != ncclInProgress) {
    set_err(KQ_ERR_BACKEND, std::string("ncclCommInitRankConfig: ") + nccl().GetErrorString(r));
    m->comm = nullptr;
    model_release(m);
    return nullptr;
  }
  if (nccl_wait(m, r, "ncclCommInitRankConfig") != KQ_OK) {
    const std::string keep = g_err;
    model_release(m);
    set_err(KQ_ERR_TIMEOUT, keep);
    return nullptr;
  }
  return m;
}

extern "C" int kq_model_tp(const kq_model* m, int* rank, int* world) {
  if (!m) return set_err(KQ_ERR_ARG, "null model");
  if (rank) *rank = m->tp_rank;
  if (world) *world = m->tp_world;
  return KQ_OK;
}

extern "C" void kq_model_free(kq_model* m) { model_release(m); }

// Synthetic stream numbering (shared specification with the CPU oracle).
static uint64_t tstream(int layer, int kind) { return (uint64_t)(layer + 1) * 32u + (uint64_t)kind; }

static int gen_normal_dev(float* dst, long long n, float mu, float sigma, uint64_t seed, uint64_t stream, cudaStream_t s) {
  k_gen_normal<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dst, n, mu, sigma, gen_base(seed, stream));
  CU(cudaGetLastError());
  return KQ_OK;
}

extern "C" int kq_model_fill_synthetic(kq_model* m, uint64_t seed) {
  int rc = model_check(m);
  if (rc) return rc;
  const kq_config& c = m->c;
  cudaStream_t s = m->stream;
  // tensor-parallel shards draw the blocks of the full matrices they slice (ShardMap)
  const int r = m->tp_rank, G = c.dim / 256, QDf = c.n_heads * c.head_dim;
  const ShardMap sq{r * m->nh_l * c.head_dim, 0, G}, skv{r * m->nkv_l * c.head_dim, 0, G};
  const ShardMap so{0, r * m->nh_l * c.head_dim / 256, QDf / 256}, sgu{r * m->ffn_l, 0, G};
  const ShardMap sdn{0, r * m->ffn_l / 256, c.ffn / 256}, sout{r * m->vocab_l, 0, G};
  for (int l = 0; l < c.n_layers; ++l) {
    LayerW& w = m->L[l];
    if ((rc = qmat_write(w.q, w.q->R, nullptr, gen_base(seed, tstream(l, KQ_T_Q)), RM_ROPE_PAIR, c.head_dim, s, sq))) return rc;
    if ((rc = qmat_write(w.k, w.k->R, nullptr, gen_base(seed, tstream(l, KQ_T_K)), RM_ROPE_PAIR, c.head_dim, s, skv))) return rc;
    if ((rc = qmat_write(w.v, w.v->R, nullptr, gen_base(seed, tstream(l, KQ_T_V)), RM_IDENT, 0, s, skv))) return rc;
    if ((rc = qmat_write(w.o, w.o->R, nullptr, gen_base(seed, tstream(l, KQ_T_O)), RM_IDENT, 0, s, so))) return rc;
    if ((rc = qmat_write(w.gu, m->ffn_l, nullptr, gen_base(seed, tstream(l, KQ_T_GATE)), RM_INTERLEAVE, 0, s, sgu))) return rc;
    if ((rc = qmat_write(w.gu, m->ffn_l, nullptr, gen_base(seed, tstream(l, KQ_T_UP)), RM_INTERLEAVE, 1, s, sgu))) return rc;
    if ((rc = qmat_write(w.down, w.down->R, nullptr, gen_base(seed, tstream(l, KQ_T_DOWN)), RM_IDENT, 0, s, sdn))) return rc;
    if ((rc = gen_normal_dev(w.attn_norm, c.dim, 1.0f, 0.02f, seed, tstream(l, KQ_T_ATTN_NORM), s))) return rc;
    if ((rc = gen_normal_dev(w.ffn_norm, c.dim, 1.0f, 0.02f, seed, tstream(l, KQ_T_FFN_NORM), s))) return rc;
  }
  if ((rc = qmat_write(m->emb, m->emb->R, nullptr, gen_base(seed, tstream(-1, KQ_T_EMB)), RM_IDENT, 0, s))) return rc;
  if ((rc = qmat_write(m->out, m->out->R, nullptr, gen_base(seed, tstream(-1, KQ_T_OUT)), RM_IDENT, 0, s, sout))) return rc;
  if ((rc = gen_normal_dev(m->out_norm, c.dim, 1.0f, 0.02f, seed, tstream(-1, KQ_T_OUTNORM), s))) return rc;
  CU(cudaStreamSynchronize(s));
  return KQ_OK;
}

static int set_tensor_impl(kq_model* m, int layer, int kind, const void* host, size_t bytes, bool pack);
extern "C" int kq_model_set_tensor(kq_model* m, int layer, int kind, const void* host, size_t bytes) {
  return set_tensor_impl(m, layer, kind, host, bytes, false);
}
static int set_tensor_impl(kq_model* m, int layer, int kind, const void* host, size_t bytes, bool pack) {
  int rc = model_check(m);
  if (rc) return rc;
  if (m->tp_world > 1) return set_err(KQ_ERR_ARG, "tensor uploads go to a whole model (tensor-parallel models are generated)");
  if (!host) return set_err(KQ_ERR_ARG, "null tensor data");
  const kq_config& c = m->c;
  const bool global = kind == KQ_T_EMB || kind == KQ_T_OUT || kind == KQ_T_OUTNORM;
  if (global != (layer < 0)) return set_err(KQ_ERR_ARG, "layer must be -1 exactly for the global tensors");
  if (!global && layer >= c.n_layers) return set_err(KQ_ERR_ARG, "layer out of range");
  float* fdst = nullptr;
  switch (kind) {
    case KQ_T_OUTNORM: fdst = m->out_norm; break;
    case KQ_T_ATTN_NORM: fdst = m->L[layer].attn_norm; break;
    case KQ_T_FFN_NORM: fdst = m->L[layer].ffn_norm; break;
    default: break;
  }
  if (fdst) {
    if (bytes != (size_t)c.dim * 4) return set_err(KQ_ERR_ARG, "norm tensors are dim float32 values");
    CU(cudaMemcpy(fdst, host, bytes, cudaMemcpyHostToDevice));
    return KQ_OK;
  }
  cudaStream_t s = m->stream;
  switch (kind) {
    case KQ_T_EMB: return qmat_upload_mapped(m->emb, host, bytes, m->emb->R, RM_IDENT, 0, s, pack);
    case KQ_T_OUT: return qmat_upload_mapped(m->out, host, bytes, m->out->R, RM_IDENT, 0, s, pack);
    case KQ_T_Q: return qmat_upload_mapped(m->L[layer].q, host, bytes, m->L[layer].q->R, RM_ROPE_PAIR, c.head_dim, s, pack);
    case KQ_T_K: return qmat_upload_mapped(m->L[layer].k, host, bytes, m->L[layer].k->R, RM_ROPE_PAIR, c.head_dim, s, pack);
    case KQ_T_V: return qmat_upload_mapped(m->L[layer].v, host, bytes, m->L[layer].v->R, RM_IDENT, 0, s, pack);
    case KQ_T_O: return qmat_upload_mapped(m->L[layer].o, host, bytes, m->L[layer].o->R, RM_IDENT, 0, s, pack);
    case KQ_T_GATE: return qmat_upload_mapped(m->L[layer].gu, host, bytes, c.ffn, RM_INTERLEAVE, 0, s, pack);
    case KQ_T_UP: return qmat_upload_mapped(m->L[layer].gu, host, bytes, c.ffn, RM_INTERLEAVE, 1, s, pack);
    case KQ_T_DOWN: return qmat_upload_mapped(m->L[layer].down, host, bytes, m->L[layer].down->R, RM_IDENT, 0, s, pack);
    default: return set_err(KQ_ERR_ARG, "unknown tensor kind");
  }
}

// ------------------------------------------------------------------------------ Kindi packs
// make_engine(pack, ctx) (engine.py:369-381): validate the pack on the host (kq_pack.h, the
// checks of verify_pack, q4pack.py:86-108), then create the model and move every tensor from the
// memory-mapped weights.bin / f32.bin to the device, the 8-row interleave regrouped on the device.
extern "C" int kq_pack_read_config(const char* dir, int ctx, kq_config* out) {
  kqpack::Pack P;
  std::string err;
  if (kqpack::read_pack(dir, ctx, P, err)) return set_err(KQ_ERR_ARG, err);
  if (validate_cfg(P.cfg) != KQ_OK) return KQ_ERR_ARG;
  if (out) *out = P.cfg;
  return KQ_OK;
}

namespace {
struct MappedFile {
  void* p = MAP_FAILED;
  size_t n = 0;
  bool open(const std::string& path, size_t size) {
    n = size;
    if (!size) return true;
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return false;
    p = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    return p != MAP_FAILED;
  }
  const uint8_t* at(uint64_t off) const { return static_cast<const uint8_t*>(p) + off; }
  ~MappedFile() { if (p != MAP_FAILED && n) ::munmap(p, n); }
};
}  // namespace

extern "C" kq_model* kq_model_load_pack(const char* dir, int ctx, int device) {
  kqpack::Pack P;
  std::string err;
  if (kqpack::read_pack(dir, ctx, P, err)) { set_err(KQ_ERR_ARG, err); return nullptr; }
  MappedFile wf, ff;
  if (!wf.open(P.dir + "/weights.bin", P.weights_size) || !ff.open(P.dir + "/f32.bin", P.f32_size)) {
    set_err(KQ_ERR_BACKEND, "cannot map the pack's weights.bin / f32.bin");
    return nullptr;
  }
  kq_model* m = model_create(&P.cfg, device, 0, 1);
  if (!m) return nullptr;
  struct Kind { const char* suffix; int kind; };
  const Kind kinds[] = {{"attn_norm.weight", KQ_T_ATTN_NORM}, {"attn_q.weight", KQ_T_Q}, {"attn_k.weight", KQ_T_K},
                        {"attn_v.weight", KQ_T_V}, {"attn_output.weight", KQ_T_O}, {"ffn_gate.weight", KQ_T_GATE},
                        {"ffn_up.weight", KQ_T_UP}, {"ffn_down.weight", KQ_T_DOWN}};
  auto put = [&](const std::string& name, int layer, int kind) -> int {
    const kqpack::Tensor& T = P.t.at(name);
    if (T.type == 0) return set_tensor_impl(m, layer, kind, ff.at(T.f32_off), (size_t)T.rows * T.cols * 4, false);
    return set_tensor_impl(m, layer, kind, wf.at(T.offset), (size_t)T.bytes, true);
  };
  int rc = put("token_embd.weight", -1, KQ_T_EMB);
  if (!rc) rc = put("output.weight", -1, KQ_T_OUT);
  if (!rc) rc = put("output_norm.weight", -1, KQ_T_OUTNORM);
  for (int l = 0; !rc && l < P.cfg.n_layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    for (const Kind& k : kinds)
      if (!rc) rc = put(p + k.suffix, l, k.kind);
    if (!rc) rc = put(p + P.ffn_norm_name, l, KQ_T_FFN_NORM);
  }
  if (!rc && cudaStreamSynchronize(m->stream) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "pack upload");
  if (rc) {
    const std::string keep = g_err;
    model_release(m);
    set_err(rc, keep);
    return nullptr;
  }
  return m;
}

extern "C" int kq_model_reset(kq_model* m) {
  int rc = model_check(m);
  if (rc) return rc;
  const size_t kvn = (size_t)m->nkv_l * m->c.head_dim * m->c.ctx;
  for (auto& l : m->L) {
    CU(cudaMemsetAsync(l.kc, 0, kvn * 2, m->stream));
    CU(cudaMemsetAsync(l.vc, 0, kvn * 2, m->stream));
  }
  CU(cudaStreamSynchronize(m->stream));
  return KQ_OK;
}

// Value of the K/V cache at (kv, pos, d) = generator element (pos * n_kv + kv) * hd + d, which is
// the element order of the reference layout [pos][kv][hd].
// A tensor-parallel rank holds heads [kv_off, kv_off + nkv) of nkv_all.
__global__ void k_fill_kv(__half* dst, int npos, int nkv, int ctx, int hd, uint64_t base, int nkv_all, int kv_off) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)npos * nkv * hd) return;
  const int d = (int)(i % hd);
  const long long r = i / hd;
  const int kv = (int)(r % nkv), pos = (int)(r / nkv);
  const uint64_t gi = ((uint64_t)pos * nkv_all + kv_off + kv) * hd + d;
  dst[((size_t)kv * ctx + pos) * hd + d] = __float2half_rn(gen_nrm(base, gi));
}

extern "C" int kq_model_fill_kv(kq_model* m, int npos, uint64_t seed) {
  int rc = model_check(m);
  if (rc) return rc;
  if (npos < 0 || npos > m->c.ctx) return set_err(KQ_ERR_ARG, "npos out of range");
  const long long n = (long long)npos * m->nkv_l * m->c.head_dim;
  if (n == 0) return KQ_OK;
  const int kv_off = m->tp_rank * m->nkv_l;
  for (int l = 0; l < m->c.n_layers; ++l) {
    k_fill_kv<<<(unsigned)((n + 255) / 256), 256, 0, m->stream>>>(m->L[l].kc, npos, m->nkv_l, m->c.ctx, m->c.head_dim,
                                                                   gen_base(seed, tstream(l, 12)), m->c.n_kv_heads, kv_off);
    k_fill_kv<<<(unsigned)((n + 255) / 256), 256, 0, m->stream>>>(m->L[l].vc, npos, m->nkv_l, m->c.ctx, m->c.head_dim,
                                                                   gen_base(seed, tstream(l, 13)), m->c.n_kv_heads, kv_off);
  }
  CU(cudaGetLastError());
  CU(cudaStreamSynchronize(m->stream));
  return KQ_OK;
}

extern "C" int kq_model_get_kv(kq_model* m, int layer, int which, int npos, uint16_t* out) {
  int rc = model_check(m);
  if (rc) return rc;
  if (layer < 0 || layer >= m->c.n_layers || npos < 0 || npos > m->c.ctx || !out || (which != 0 && which != 1))
    return set_err(KQ_ERR_ARG, "bad K/V cache request");
  const int nkv = m->nkv_l, hd = m->c.head_dim, ctx = m->c.ctx;   // this rank's heads
  std::vector<uint16_t> tmp((size_t)nkv * ctx * hd);
  CU(cudaMemcpy(tmp.data(), which ? m->L[layer].vc : m->L[layer].kc, tmp.size() * 2, cudaMemcpyDeviceToHost));
  for (int p = 0; p < npos; ++p)
    for (int kv = 0; kv < nkv; ++kv)
      std::memcpy(out + ((size_t)p * nkv + kv) * hd, tmp.data() + ((size_t)kv * ctx + p) * hd, hd * 2);
  return KQ_OK;
}

// ------------------------------------------------------------------------------ decode step
// One token as a list of operations: per layer qkv / attention / o / gate-up / down, then the
// head. `persist` selects the launch shapes of the persistent kernel instead of the per-kernel
// planner; the buffers and fusions are the same.
struct StepOp {
  int kind;              // PH_GEMV / PH_ATTN
  GemvParams g;
  GemvPlan pl;           // per-kernel launches only
  int stage_bytes;       // persistent kernel only
  AttnSplitParams a;
  bool tmv;              // per-kernel launches: this GEMV runs as k_tmv (t, tgrid)
  TmvParams t;
  dim3 tgrid;
};

// The tensor-core GEMV form of a decode GEMV: the same segments, activation source and
// epilogues; one CTA per SM over the (128-row tile, super-block) units. `part` holds nsm * 2 * 128
// floats and `ticket` TV_MAX_TILES ints (zero). False when the launch is not covered (embedding
// prologue, argmax epilogue, more than TV_MAX_G super-blocks per row, shared memory) or the
// tensor-core GEMV is off: k_gemv runs it.
static bool tmv_plan(const GemvParams& g, int nsm, size_t smem_max, float* part, int* ticket, TmvParams& T, dim3& grid) {
  if (smem_max == 0 || g.nseg < 1 || g.nseg > TV_MAX_SEG || g.G > TV_MAX_G) return false;
  if (g.xmode != XS_PLAIN && g.xmode != XS_NORM) return false;
  std::memset(&T, 0, sizeof(T));
  int ntiles = 0;
  for (int i = 0; i < g.nseg; ++i) {
    const Seg& sg = g.seg[i];
    if (sg.epi == EPI_ARGMAX || sg.w.G != g.G || !sg.w.tv) return false;
    T.seg[i].w = sg.w;
    T.seg[i].tile0 = ntiles;
    T.seg[i].epi = sg.epi;
    T.seg[i].out_f = sg.out_f;
    T.seg[i].out_h = sg.out_h;
    ntiles += (sg.w.R + TV_ROWS - 1) / TV_ROWS;
    if (sg.w.type == Q4K) T.has_q4 = 1;
    else T.has_q6 = 1;
  }
  if (ntiles > TV_MAX_TILES) return false;
  const size_t smem = tv_smem(g.G, T.has_q4 != 0, T.has_q6 != 0).total;
  if (smem > smem_max) return false;
  T.nseg = g.nseg;
  T.ntiles = ntiles;
  T.G = g.G;
  T.smem = (int)smem;
  T.xmode = g.xmode;
  T.x = g.x;
  T.h_in = g.h_in;
  T.y_add = g.y_add;
  T.gamma = g.gamma;
  T.h_out = g.h_out;
  T.eps = g.eps;
  T.st = g.st;
  T.cos_t = g.cos_t;
  T.sin_t = g.sin_t;
  T.hd = g.hd;
  T.ctx = g.ctx;
  T.part = part;
  T.ticket = ticket;
  T.err = g.err;
  const long long U = (long long)ntiles * g.G;
  grid = dim3((unsigned)std::min<long long>(nsm, U));
  return true;
}

static int build_step(kq_model* m, bool head, bool persist, std::vector<StepOp>& ops) {
  const kq_config& c = m->c;
  int trace = 0;   // launch index within the step (phase trace of KQ_TRACE builds)
  int ngemv = 0;   // GEMV launches so far: each has its own stage-claim counters
  ops.clear();
  int cur = 0;
  auto gemv = [&](const SegSpec* ss, int nseg, bool pairs, StepOp& op) -> int {
    op.kind = PH_GEMV;
    op.tmv = false;
    op.stage_bytes = 0;
    int rc = persist ? fill_gemv_dec(ss, nseg, op.g, op.stage_bytes) : fill_gemv(ss, nseg, pairs, m->nsm, op.g, op.pl);
    if (rc) return rc;
    GemvParams& pp = op.g;
    pp.st = m->st;
    pp.vocab = c.vocab;
    // the rotary tables only where an epilogue rotates (the q/k/v GEMV); elsewhere the prologue
    // would wait on loads it does not need
    bool rope = false;
    for (int i = 0; i < nseg; ++i) rope |= ss[i].epi == EPI_ROPE_Q || ss[i].epi == EPI_ROPE_K;
    pp.cos_t = rope ? m->cos_t : nullptr;
    pp.sin_t = rope ? m->sin_t : nullptr;
    pp.hd = c.head_dim;
    pp.ctx = c.ctx;
    pp.err = m->err;
    pp.eps = c.eps;
    pp.trace_id = trace++;
    // run-time stage claims for launches of at least 3 stages per CTA (gate/up, down, head; the
    // short q/k/v and o launches keep fixed ranges, which balance better at 1-2 stages a CTA).
    // The launches of one step run in stream order, and the same launch of the next step only
    // after this one finished, so a counter pair per launch suffices. Switch: KQ_GEMV_DYN=0
    if (!persist && m->gdyn && ngemv < KQ_MAX_STEP_GEMVS && pp.nstages >= 3 * op.pl.grid) pp.dyn = m->gdyn + 2 * ngemv;
    ++ngemv;
    return KQ_OK;
  };
  for (int l = 0; l < c.n_layers; ++l) {
    LayerW& w = m->L[l];
    StepOp op;
    // QKV (+ norm or embedding; rotary + K/V store)
    SegSpec qkv[3] = {{w.q, EPI_ROPE_Q, m->q, nullptr}, {w.k, EPI_ROPE_K, nullptr, w.kc}, {w.v, EPI_V, nullptr, w.vc}};
    int rc = gemv(qkv, 3, true, op);
    if (rc) return rc;
    GemvParams& p = op.g;
    if (l == 0) {
      p.xmode = XS_EMBED;
      p.emb = m->emb->view();
      p.h_in = nullptr;
      p.y_add = nullptr;
    } else {
      p.xmode = XS_NORM;
      p.h_in = m->h[cur];
      p.y_add = m->y;
    }
    p.gamma = w.attn_norm;
    p.h_out = m->h[cur ^ 1];
    cur ^= 1;
    ops.push_back(op);
    // attention
    StepOp at{};
    at.kind = PH_ATTN;
    AttnParams& a = at.a.a;
    a.q = m->q; a.kc = w.kc; a.vc = w.vc;
    a.out = m->att; a.st = m->st; a.n_kv = c.n_kv_heads; a.ctx = c.ctx;
    a.scale = (float)(1.0 / std::sqrt((double)c.head_dim));
    a.err = m->err;
    a.trace_id = trace++;
    at.a.part = m->apart;
    at.a.part_ml = m->apart_ml;
    at.a.ticket = m->aticket;
    at.a.nsplit = m->attn_nsplit;
    ops.push_back(at);
    // o projection
    SegSpec so[1] = {{w.o, EPI_F32, m->y, nullptr}};
    if ((rc = gemv(so, 1, false, op))) return rc;
    op.g.xmode = XS_PLAIN;
    op.g.x = m->att;
    ops.push_back(op);
    // gate/up (+ norm, SwiGLU)
    SegSpec sg[1] = {{w.gu, EPI_SWIGLU, m->mbuf, nullptr}};
    if ((rc = gemv(sg, 1, true, op))) return rc;
    op.g.xmode = XS_NORM;
    op.g.h_in = m->h[cur];
    op.g.y_add = m->y;
    op.g.gamma = w.ffn_norm;
    op.g.h_out = m->h[cur ^ 1];
    cur ^= 1;
    ops.push_back(op);
    // down
    SegSpec sd[1] = {{w.down, EPI_F32, m->y, nullptr}};
    if ((rc = gemv(sd, 1, false, op))) return rc;
    op.g.xmode = XS_PLAIN;
    op.g.x = m->mbuf;
    ops.push_back(op);
  }
  if (head) {
    StepOp op;
    SegSpec sh[1] = {{m->out, EPI_ARGMAX, m->logits, nullptr}};
    int rc = gemv(sh, 1, false, op);
    if (rc) return rc;
    if (!persist && op.pl.grid > 1024) return set_err(KQ_ERR_ARG, "head grid too large");
    GemvParams& p = op.g;
    p.xmode = XS_NORM;
    p.h_in = m->h[cur];
    p.y_add = m->y;
    p.gamma = m->out_norm;
    p.h_out = m->h[cur ^ 1];
    p.part_val = m->hpart_val;
    p.part_idx = m->hpart_idx;
    p.ticket = m->hticket;
    p.out_ids = m->out_ids;
    p.out_cap = m->out_cap;
    ops.push_back(op);
  }
  if (!persist)
    for (StepOp& op : ops)
      if (op.kind == PH_GEMV)
        op.tmv = !op.pl.mma && tmv_plan(op.g, m->nsm, g_dev[m->device].tmv_smem, m->tv_part, m->tv_ticket, op.t, op.tgrid);
  return KQ_OK;
}

// A launch that may start while the previous kernel on the stream finishes (it waits in-kernel);
// pdl = false: an ordinary launch that starts after the previous work on the stream.
template <class K, class PT>
static cudaError_t launch_pdl(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const PT& p, bool pdl = true) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}
// Decode attention on the tensor cores: grid (token, KV head, split), merge per (token, KV head).
template <int G>
static cudaError_t launch_dattn_t(const DAttnParams& P, int M, int nkv, cudaStream_t s) {
  cudaError_t e = launch_pdl(k_dattn_mma<G>, dim3((unsigned)M, (unsigned)nkv, (unsigned)P.nsplit), dim3(32), DM_SMEM, s, P);
  if (e != cudaSuccess) return e;
  return launch_pdl(k_dattn_merge<G>, dim3((unsigned)M, (unsigned)nkv, (unsigned)G), dim3(DM_MERGE_THREADS), 0, s, P);
}

// The step's first kernel (the q/k/v GEMV that embeds the token) is launched without the PDL
// attribute: the GEMV prologues read the step state (token, position) before their dependency
// wait, which is only safe when the host's state upload has completed before the kernel starts.
// Every later kernel reads state that an earlier kernel of the same step does not write.
static int enqueue_step(kq_model* m, bool head, cudaStream_t s) {
  std::vector<StepOp> ops;
  int rc = build_step(m, head, false, ops);
  if (rc) return rc;
  const int G = m->c.n_heads / m->c.n_kv_heads;
  bool first = true;
  for (const StepOp& op : ops) {
    if (op.kind == PH_GEMV) {
      if (op.tmv) CU(launch_pdl(k_tmv, op.tgrid, dim3(TV_THREADS), (size_t)op.t.smem, s, op.t, !first));
      else CU(launch_gemv(op.g, op.pl, s, !first));
    } else if (m->attn_mode == 1) {
      CU(attn_cl_fn(G, m->attn_cl)(op.a.a, s, true));
    } else if (m->attn_mode == 2) {
      DAttnParams D;
      std::memset(&D, 0, sizeof(D));
      D.q = op.a.a.q; D.kc = op.a.a.kc; D.vc = op.a.a.vc; D.st = op.a.a.st; D.err = op.a.a.err;
      D.n_kv = op.a.a.n_kv; D.ctx = op.a.a.ctx; D.scale = op.a.a.scale;
      D.nsplit = m->dsplit; D.part = m->dpart1; D.out_f = op.a.a.out; D.trace_id = op.a.a.trace_id;
      CU(G == 1 ? launch_dattn_t<1>(D, 1, D.n_kv, s) : G == 2 ? launch_dattn_t<2>(D, 1, D.n_kv, s)
         : G == 4 ? launch_dattn_t<4>(D, 1, D.n_kv, s) : launch_dattn_t<8>(D, 1, D.n_kv, s));
    } else {
      CU(launch_attn_split(op.a, G, s, true));
    }
    first = false;
  }
  return KQ_OK;
}

// ------------------------------------------------------------------------------ persistent kernel
typedef cudaError_t (*DecFn)(const DecodeParams&, int grid, size_t smem, cudaStream_t s);
template <int G>
static cudaError_t launch_decode_t(const DecodeParams& d, int grid, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(DEC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;   // every CTA resident at once, or the launch fails
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_decode<G>, d);
}
static const void* decode_fn_ptr(int G) {
  return G == 1 ? (const void*)k_decode<1> : G == 2 ? (const void*)k_decode<2> : G == 4 ? (const void*)k_decode<4>
                                                                                       : (const void*)k_decode<8>;
}
static DecFn decode_fn(int G) {
  return G == 1 ? launch_decode_t<1> : G == 2 ? launch_decode_t<2> : G == 4 ? launch_decode_t<4> : launch_decode_t<8>;
}

// Builds the phase table and the launch shape of the persistent kernel (once per model).
static int setup_persistent(kq_model* m) {
  std::vector<StepOp> ops;
  int rc = build_step(m, true, true, ops);
  if (rc) return rc;
  const int G = m->c.n_heads / m->c.n_kv_heads;
  size_t slot = (size_t)2 * ATT_P * 128 * 2;   // one K + V chunk
  size_t work = 0;
  for (const StepOp& op : ops) {
    if (op.kind == PH_GEMV) {
      const int nthr_c = op.g.LPR * op.g.NRG * op.g.nlanes;
      if (op.g.xmode != XS_PLAIN && 8 * op.g.LPR > 2 * nthr_c)
        return set_err(KQ_ERR_ARG, "persistent kernel: a normed GEMV input is too wide (more than 2 items per thread)");
      slot = std::max(slot, (size_t)op.stage_bytes);
      work = std::max(work, gemv_smem_layout(0, 0, op.g.LPR, op.g.NRG * op.g.nlanes, DEC_RPG, nthr_c).total);
    }
  }
  const size_t att_work = (size_t)(G == 1 ? AttnScratch<1>::total : G == 2 ? AttnScratch<2>::total
                                   : G == 4 ? AttnScratch<4>::total : AttnScratch<8>::total) * 4;
  work = align_up(std::max(work, att_work), 128);
  slot = align_up(slot, 128);
  const size_t desc = align_up(DEC_NDESC * sizeof(PhaseDesc), 128);
  cudaFuncAttributes fa;
  CU(cudaFuncGetAttributes(&fa, decode_fn_ptr(G)));
  int optin = 0;
  CU(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
  const size_t budget = (size_t)optin - fa.sharedSizeBytes;
  const size_t fixed = work + desc + (2 * DEC_NB + DEC_NDESC) * 8;
  if (budget < fixed + 2 * slot) return set_err(KQ_ERR_ARG, "persistent kernel does not fit in shared memory");
  const size_t ring = (budget - fixed) / 128 * 128;   // >= 2 largest entries (checked above)
  DecodeParams& d = m->dec;
  std::memset(&d, 0, sizeof(d));
  d.ring_bytes = (int)ring;
  d.work_off = (int)ring;
  d.desc_off = (int)(d.work_off + work);
  d.bars_off = (int)(d.desc_off + desc);
  m->dec_smem = (size_t)d.bars_off + (size_t)(2 * DEC_NB + DEC_NDESC) * 8;
  CU(cudaFuncSetAttribute(decode_fn_ptr(G), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->dec_smem));
  // phase table on the device
  std::vector<PhaseDesc> ph(ops.size());
  std::memset(ph.data(), 0, ph.size() * sizeof(PhaseDesc));
  for (size_t i = 0; i < ops.size(); ++i) {
    ph[i].kind = ops[i].kind;
    if (ops[i].kind == PH_GEMV) ph[i].g = ops[i].g;
    else ph[i].a = ops[i].a;
  }
  bool ok = true;
  m->d_phases = dalloc<PhaseDesc>(m, ph.size(), ok);
  m->nph_all = (int)ph.size();
  m->dec_bar = dalloc<int>(m, ph.size() + 1, ok);
  if (!ok) return set_err(KQ_ERR_MEMORY, "persistent kernel tables");
  CU(cudaMemcpy(m->d_phases, ph.data(), ph.size() * sizeof(PhaseDesc), cudaMemcpyHostToDevice));
  d.ph = m->d_phases;
  d.bar = m->dec_bar;
  d.nbar = m->nph_all + 1;
  d.st = m->st;
  d.err = m->err;
  // the whole grid must be co-resident: one CTA per SM
  int per_sm = 0;
  CU(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_fn_ptr(G), DEC_THREADS, m->dec_smem));
  if (per_sm < 1) return set_err(KQ_ERR_BACKEND, "persistent decode kernel cannot be resident");
  if (std::getenv("KQ_VERBOSE"))
    std::fprintf(stderr, "kq: persistent decode: %d phases, ring %zu B (largest stage %zu B), work %zu B, smem %zu B\n",
                 m->nph_all, ring, slot, work, m->dec_smem);
  return KQ_OK;
}

static int launch_persistent(kq_model* m, bool head) {
  DecodeParams d = m->dec;
  d.nph = head ? m->nph_all : m->nph_all - 1;
  const int G = m->c.n_heads / m->c.n_kv_heads;
  CU(decode_fn(G)(d, m->nsm, m->dec_smem, m->stream));
  return KQ_OK;
}

static int build_graph(kq_model* m, bool head, cudaGraphExec_t* out) {
  cudaGraph_t g = nullptr;
  CU(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_step(m, head, m->stream);
  cudaError_t e = cudaStreamEndCapture(m->stream, &g);
  if (rc) { if (g) cudaGraphDestroy(g); return rc; }
  if (e != cudaSuccess) return set_err(KQ_ERR_BACKEND, std::string("graph capture: ") + cudaGetErrorString(e));
  size_t nn = 0;
  if (head && cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess) {   // kernels of one decode step
    std::vector<cudaGraphNode_t> nodes(nn);
    int kernels = 0;
    if (nn && cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
      for (cudaGraphNode_t n : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(n, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
      }
    m->step_kernels = kernels;
  }
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return set_err(KQ_ERR_BACKEND, std::string("graph instantiate: ") + cudaGetErrorString(e));
  return KQ_OK;
}

static int ensure_graphs(kq_model* m) {
  int rc;
  if (m->persist) return m->d_phases ? KQ_OK : setup_persistent(m);
  if (!m->g_step && (rc = build_graph(m, true, &m->g_step))) return rc;
  if (!m->g_feed && (rc = build_graph(m, false, &m->g_feed))) return rc;
  return KQ_OK;
}

static int check_dev_err(kq_model* m) {
  int e = 0;
  CU(cudaMemcpy(&e, m->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    cudaMemset(m->err, 0, sizeof(int));
    if (m->dec_bar) cudaMemset(m->dec_bar, 0, (size_t)(m->nph_all + 1) * sizeof(int));   // re-arm the phase counters
    if (e & (KQ_DEV_ERR_BAD_TOKEN | KQ_DEV_ERR_BAD_POS)) return set_err(KQ_ERR_ARG, "device saw an invalid token or position");
    char buf[96];
    std::snprintf(buf, sizeof buf, "a bounded device wait gave up (error bits 0x%x)", e);
    return set_err(KQ_ERR_TIMEOUT, buf);
  }
  return KQ_OK;
}

// A plain decode step's state: slot = rotary position = pos, every slot up to pos attended.
static void plain_state(DecodeState* st, int tok, int pos) {
  std::memset(st, 0, sizeof(*st));
  st->tok = tok;
  st->pos = pos;
  st->next_tok = -1;
  st->rpos = pos;
  st->tree_base = pos + 1;
}

static int run_one(kq_model* m, int tok, int pos, bool head) {
  int rc = model_check(m);
  if (rc) return rc;
  if (tok < 0 || tok >= m->c.vocab || pos < 0) return set_err(KQ_ERR_ARG, "Invalid token or position");
  if (pos >= m->c.ctx) return set_err(KQ_ERR_OVERFLOW, "position is past the context");
  if ((rc = ensure_graphs(m))) return rc;
  plain_state(m->st_host, tok, pos);
  CU(cudaMemcpyAsync(m->st, m->st_host, sizeof(DecodeState), cudaMemcpyHostToDevice, m->stream));
  if (m->persist) {
    if ((rc = launch_persistent(m, head))) return rc;
  } else {
    CU(cudaGraphLaunch(head ? m->g_step : m->g_feed, m->stream));
  }
  if (head) CU(cudaMemcpyAsync(m->st_host, m->st, sizeof(DecodeState), cudaMemcpyDeviceToHost, m->stream));
  CU(cudaStreamSynchronize(m->stream));
  if ((rc = check_dev_err(m))) return rc;
  return head ? m->st_host->next_tok : KQ_OK;
}

extern "C" int kq_verify(kq_model* m, const int32_t* tokens, const int32_t* parents, int n, int pos, float* logits,
                         int32_t* best);
extern "C" int kq_feed_batch(kq_model* m, const int32_t* toks, int n, int pos);

// A tensor-parallel model runs every token through the batched pass (a one-node pass for a
// decode step); the whole model uses the decode graph.
extern "C" int kq_feed(kq_model* m, int tok, int pos) {
  if (m && m->tp_world > 1) return kq_feed_batch(m, &tok, 1, pos);
  return run_one(m, tok, pos, false);
}
extern "C" int kq_step(kq_model* m, int tok, int pos) {
  if (m && m->tp_world > 1) {
    const int32_t par = -1;
    int32_t best = -1;
    const int rc = kq_verify(m, &tok, &par, 1, pos, nullptr, &best);
    return rc < 0 ? rc : best;
  }
  return run_one(m, tok, pos, true);
}
static int not_tp(kq_model* m, const char* what) {
  if (m && m->tp_world > 1) return set_err(KQ_ERR_ARG, std::string(what) + " runs on a whole model, not a tensor-parallel shard");
  return KQ_OK;
}

static int verify_buffers(kq_model* m);
static int batch_buffers(kq_model* m);
static bool batch_supported(const kq_model* m);
static int verify_pass(kq_model* m, const int32_t* tokens, int b0, int b1, int pos, const int* depth,
                       const unsigned long long (*anc)[2], bool head = true, int seq = -1);
static int head_argmax(kq_model* m, int M, const BatchParams& B, int* out_ids, size_t row0 = 0);

// Ancestor masks of a linear chain of MM_MAXM tokens: token j attends to tokens 0..j.
struct ChainMasks {
  int depth[MM_MAXM];
  unsigned long long anc[MM_MAXM][2];
  ChainMasks() {
    for (int j = 0; j < MM_MAXM; ++j) {
      depth[j] = j;
      anc[j][0] = j >= 63 ? ~0ull : ((1ull << (j + 1)) - 1);
      anc[j][1] = j < 64 ? 0ull : j == 127 ? ~0ull : ((1ull << (j - 63)) - 1);
    }
  }
};

// Prefill (Engine.feed_batch, gpu4.py:109-110 feeds token by token): chunks of up to MM_MAXM
// tokens run as batched passes on the tensor cores, each chunk a linear chain whose token j
// attends to the positions below the chunk and to chunk tokens 0..j; K/V only, no head. A single
// token, and configurations the batched pass does not cover, take the decode step.
extern "C" int kq_feed_batch(kq_model* m, const int32_t* toks, int n, int pos) {
  int rc = model_check(m);
  if (rc) return rc;
  if (!toks || n < 0 || pos < 0) return set_err(KQ_ERR_ARG, "bad token batch");
  for (int i = 0; i < n; ++i)
    if (toks[i] < 0 || toks[i] >= m->c.vocab) return set_err(KQ_ERR_ARG, "Invalid token");
  if (pos + n > m->c.ctx) return set_err(KQ_ERR_OVERFLOW, "prompt runs past the context");
  if (m->tp_world == 1 && (n < 2 || m->verify_seq || !batch_supported(m))) {
    for (int i = 0; i < n; ++i)
      if ((rc = kq_feed(m, toks[i], pos + i)) < 0) return rc;
    return KQ_OK;
  }
  if ((m->tp_world == 1 && (rc = ensure_graphs(m))) || (rc = verify_buffers(m)) || (rc = batch_buffers(m))) return rc;
  static const ChainMasks chain;
  for (int c0 = 0; c0 < n; c0 += MM_MAXM)
    if ((rc = verify_pass(m, toks + c0, 0, std::min(MM_MAXM, n - c0), pos + c0, chain.depth, chain.anc, false)))
      return rc;
  prof_mark(m, PC_END);
  if ((rc = tp_sync(m))) return rc;
  prof_flush(m);
  return check_dev_err(m);
}

extern "C" int kq_generate(kq_model* m, const int32_t* ids, int n_ids, int n, int32_t* out) {
  if (!ids || n_ids < 1 || n < 1 || !out) return set_err(KQ_ERR_ARG, "bad generate arguments");
  int rc = kq_model_reset(m);
  if (rc) return rc;
  if ((rc = kq_feed_batch(m, ids, n_ids - 1, 0))) return rc;
  int pos = n_ids;
  int t = kq_step(m, ids[n_ids - 1], pos - 1);
  if (t < 0) return t;
  out[0] = t;
  for (int i = 1; i < n; ++i) {
    t = kq_step(m, out[i - 1], pos);
    if (t < 0) return t;
    out[i] = t;
    ++pos;
  }
  return KQ_OK;
}

extern "C" int kq_logits(kq_model* m, int row, float* out) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "kq_logits"))) return rc;
  if (row != 0 || !out) return set_err(KQ_ERR_ARG, "bad logits request");
  CU(cudaMemcpy(out, m->logits, (size_t)m->c.vocab * 4, cudaMemcpyDeviceToHost));
  return KQ_OK;
}

extern "C" int kq_hidden(kq_model* m, float* out) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "kq_hidden"))) return rc;
  if (!out) return set_err(KQ_ERR_ARG, "null output");
  // after a step with the head, the residual (h + last block output) is in h[1] (even number of
  // norm kernels per layer, the head's norm writes the second buffer)
  CU(cudaMemcpy(out, m->h[1], (size_t)m->c.dim * 4, cudaMemcpyDeviceToHost));
  return KQ_OK;
}

extern "C" int kq_decode_loop(kq_model* m, int tok, int pos, int n, int32_t* out) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "kq_decode_loop"))) return rc;
  if (n < 1 || !out || tok < 0 || tok >= m->c.vocab || pos < 0) return set_err(KQ_ERR_ARG, "bad decode loop arguments");
  if (pos + n > m->c.ctx) return set_err(KQ_ERR_OVERFLOW, "decode loop runs past the context");
  if ((rc = ensure_graphs(m))) return rc;
  if (n > m->out_cap) return set_err(KQ_ERR_ARG, "decode loop longer than the context");
  plain_state(m->st_host, tok, pos);
  CU(cudaMemcpyAsync(m->st, m->st_host, sizeof(DecodeState), cudaMemcpyHostToDevice, m->stream));
  // each replay embeds st->tok at st->pos; the head's last CTA stores the argmax in out_ids and
  // advances (tok, pos) on the device, so no host round trip separates the steps
  for (int i = 0; i < n; ++i) {
    if (m->persist) {
      if ((rc = launch_persistent(m, true))) return rc;
    } else {
      CU(cudaGraphLaunch(m->g_step, m->stream));
    }
  }
  CU(cudaMemcpyAsync(out, m->out_ids, (size_t)n * sizeof(int32_t), cudaMemcpyDeviceToHost, m->stream));
  CU(cudaStreamSynchronize(m->stream));
  return check_dev_err(m);
}

extern "C" int kq_phase_times(kq_model* m, float* ms4) {
  int rc = model_check(m);
  if (rc) return rc;
  if (!ms4) return set_err(KQ_ERR_ARG, "null output");
  if (!m->prof) return set_err(KQ_ERR_ARG, "the time split is off (set KQ_PHASE_TIMES=1 before creating the model)");
  for (int i = 0; i < 4; ++i) {
    ms4[i] = (float)m->pms[i];
    m->pms[i] = 0.0;
  }
  return KQ_OK;
}

extern "C" int kq_step_kernels(kq_model* m) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "kq_step_kernels"))) return rc;
  if ((rc = ensure_graphs(m))) return rc;
  return m->persist ? 1 : m->step_kernels;
}

extern "C" int kq_time_decode(kq_model* m, int tok, int pos, int n, float* ms_out) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "kq_time_decode"))) return rc;
  if (n < 1 || !ms_out || tok < 0 || tok >= m->c.vocab || pos < 0) return set_err(KQ_ERR_ARG, "bad timing arguments");
  if (pos + n > m->c.ctx) return set_err(KQ_ERR_OVERFLOW, "timed decode runs past the context");
  if ((rc = ensure_graphs(m))) return rc;
  plain_state(m->st_host, tok, pos);
  CU(cudaMemcpyAsync(m->st, m->st_host, sizeof(DecodeState), cudaMemcpyHostToDevice, m->stream));
  cudaEvent_t e0, e1;
  CU(cudaEventCreate(&e0));
  CU(cudaEventCreate(&e1));
  CU(cudaStreamSynchronize(m->stream));
  CU(cudaEventRecord(e0, m->stream));
  for (int i = 0; i < n; ++i) {
    if (m->persist) {
      if ((rc = launch_persistent(m, true))) return rc;
    } else {
      CU(cudaGraphLaunch(m->g_step, m->stream));
    }
  }
  CU(cudaEventRecord(e1, m->stream));
  CU(cudaEventSynchronize(e1));
  float ms = 0.f;
  CU(cudaEventElapsedTime(&ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *ms_out = ms;
  return check_dev_err(m);
}

// ------------------------------------------------------------------------------ speculative verification
// Node depths and ancestor masks of a draft tree (parents[0] = -1, 0 <= parents[i] < i).
static int tree_check(const int32_t* parents, int n, int* depth, unsigned long long (*anc)[2]) {
  if (!parents || n < 1 || n > KQ_MAX_TREE || parents[0] != -1) return set_err(KQ_ERR_ARG, "bad draft tree");
  for (int i = 0; i < n; ++i) {
    if (i > 0 && (parents[i] < 0 || parents[i] >= i)) return set_err(KQ_ERR_ARG, "bad draft tree: parents[i] must lie in [0, i)");
    depth[i] = i ? depth[parents[i]] + 1 : 0;
    anc[i][0] = i ? anc[parents[i]][0] : 0;
    anc[i][1] = i ? anc[parents[i]][1] : 0;
    anc[i][i >> 6] |= 1ull << (i & 63);
  }
  return KQ_OK;
}

static int verify_buffers(kq_model* m) {
  if (m->vlogits) return KQ_OK;
  bool ok = true;
  const size_t V = (size_t)m->c.vocab;
  m->vlogits = dalloc<float>(m, KQ_MAX_TREE * V, ok);
  m->ap = dalloc<float>(m, V, ok);
  m->aq = dalloc<float>(m, V, ok);
  m->ag = dalloc<float>(m, KQ_MAX_TREE * V, ok);
  m->atok = dalloc<int>(m, KQ_MAX_TREE + 1, ok);
  m->apar = dalloc<int>(m, KQ_MAX_TREE + 1, ok);
  m->apath = dalloc<int>(m, KQ_MAX_TREE + 1, ok);
  m->aout = dalloc<int>(m, KQ_MAX_TREE + 1, ok);
  m->acnt = dalloc<int>(m, 2, ok);
  m->agrid = dalloc<AccGridScratch>(m, 1, ok);
  m->auacc = dalloc<float>(m, KQ_MAX_TREE, ok);
  m->aufin = dalloc<float>(m, KQ_MAX_TREE, ok);
  m->caches = dalloc<__half*>(m, 2 * (size_t)m->c.n_layers, ok);
  if (ok && cudaMallocHost(&m->vstates, KQ_MAX_TREE * sizeof(DecodeState)) != cudaSuccess) ok = false;
  if (!ok) return set_err(KQ_ERR_MEMORY, "verify buffers");
  std::vector<__half*> cp(2 * (size_t)m->c.n_layers);
  for (int l = 0; l < m->c.n_layers; ++l) { cp[2 * l] = m->L[l].kc; cp[2 * l + 1] = m->L[l].vc; }
  CU(cudaMemcpy(m->caches, cp.data(), cp.size() * sizeof(__half*), cudaMemcpyHostToDevice));
  return KQ_OK;
}

// ------------------------------------------------------------------------------ tensor-core GEMM
// Split-K factor: the fewest waves x super-blocks per CTA (plus a fixed per-CTA cost of about two
// super-blocks: set-up, pipeline fill, epilogue), over splits of 1..16.
static int tmm_split(int ntiles, int G, int nsm) {
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= std::min(G, 16); ++s) {
    const long long ctas = (long long)ntiles * s, waves = (ctas + nsm - 1) / nsm;
    const long long cost = waves * ((G + s - 1) / s + 2);
    if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = s; }
  }
  return best;
}
// Comparison switch: KQ_TMM_EXACT=0 keeps every row tile on the split-weight form (the exact form
// needs the sub-block sums of the packed input and Npad <= 64; it covers Q4_K row tiles).
static bool tmm_exact_ok() {
  const char* e = std::getenv("KQ_TMM_EXACT");
  return !(e && std::atoi(e) == 0);
}
static int tmm_tiles(const SegSpec* ss, int nseg) {
  int t = 0;
  for (int i = 0; i < nseg; ++i) t += (ss[i].m->R + TM_ROWS - 1) / TM_ROWS;
  return t;
}
// Segments, tiles and split of one GEMM over M tokens (outputs and scratch filled by the caller).
static void tmm_fill(const SegSpec* ss, int nseg, int M, int device, TmmParams& P) {
  const int nsm = g_dev[device].nsm;
  std::memset(&P, 0, sizeof(P));
  int tiles = 0;
  for (int i = 0; i < nseg; ++i) {
    P.seg[i].w = ss[i].m->view();
    P.seg[i].epi = ss[i].epi;
    P.seg[i].tile0 = tiles;
    P.seg[i].out_f = ss[i].out_f;
    P.seg[i].out_h = ss[i].out_h;
    tiles += (ss[i].m->R + TM_ROWS - 1) / TM_ROWS;
  }
  P.nseg = nseg;
  P.ntiles = tiles;
  P.C = ss[0].m->C;
  P.G = P.C / 256;
  P.M = M;
  P.Npad = (M + 15) & ~15;
  P.nsplit = tmm_split(tiles, P.G, nsm);
  P.xs = tmm_xs(P.Npad, g_dev[device].tmm_budget);
}
static size_t tmm_part_floats(int ntiles, int nsplit, int Npad) {
  return nsplit > 1 ? (size_t)nsplit * Npad * ntiles * TM_ROWS : 0;
}
static cudaError_t tmm_launch(const TmmParams& P, cudaStream_t s, bool pdl) {
  if (P.xs < 1 || P.Npad > TM_MAXN) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)P.ntiles, (unsigned)P.nsplit);
  cfg.blockDim = dim3(TM_THREADS);
  cfg.dynamicSmemBytes = tmm_smem(P.Npad, P.xs);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_tmm, P);
}

// Sum of the row-split GEMM partials over the tensor-parallel ranks (fp32, in place, on the
// model's stream). World 1: nothing.
static int tp_allreduce(kq_model* m, float* buf, size_t n) {
  if (m->tp_world == 1) return KQ_OK;
  prof_mark(m, PC_COMM);
  int rc = tp_alive(m);
  if (rc) return rc;
  return nccl_wait(m, nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum, m->comm, m->stream), "ncclAllReduce");
}

static int batch_buffers(kq_model* m) {
  if (m->bh) return KQ_OK;
  const kq_config& c = m->c;
  const size_t MM = MM_MAXM, QD = (size_t)m->nh_l * c.head_dim;   // this rank's heads
  bool ok = true;
  m->bh = dalloc<float>(m, MM * c.dim, ok);
  m->by = dalloc<float>(m, MM * c.dim, ok);
  m->bq = dalloc<float>(m, MM * QD, ok);
  m->bxd = dalloc<__half>(m, xp_halves(MM_MAXM, c.dim), ok);
  m->bxa = dalloc<__half>(m, xp_halves(MM_MAXM, (int)QD), ok);
  m->bxf = dalloc<__half>(m, xp_halves(MM_MAXM, m->ffn_l), ok);
  m->bxs_n = dalloc<float>(m, MM, ok);
  m->bxs_f = dalloc<float>(m, MM, ok);
  if (c.dim % 256 == 0) m->bxd_sum = dalloc<float>(m, MM * (c.dim / 32), ok);
  if (m->ffn_l % 256 == 0) m->bxf_sum = dalloc<float>(m, MM * (m->ffn_l / 32), ok);
  m->bmf = dalloc<float>(m, MM * m->ffn_l, ok);
  m->btok = dalloc<int>(m, MM, ok);
  m->bslot = dalloc<int>(m, MM, ok);
  m->brpos = dalloc<int>(m, MM, ok);
  m->bmask = dalloc<unsigned long long>(m, 2 * MM, ok);
  // attention: key splits of up to 32, row groups of BA_ROWS query rows
  const int G = c.n_heads / c.n_kv_heads, rowgroups = (MM_MAXM * G + BA_ROWS - 1) / BA_ROWS;
  m->b_nsplit = BA_MAX_SPLIT;
  m->bpart = dalloc<float>(m, (size_t)m->nkv_l * rowgroups * m->b_nsplit * BA_ROWS * BA_PLD, ok);
  m->bticket = dalloc<int>(m, (size_t)m->nkv_l * rowgroups, ok);
  // GEMM split-K scratch: the largest of the pass's GEMMs
  const LayerW& w = m->L[0];
  const SegSpec qkv[3] = {{w.q, 0, nullptr, nullptr}, {w.k, 0, nullptr, nullptr}, {w.v, 0, nullptr, nullptr}};
  const SegSpec one[4] = {{w.o, 0, nullptr, nullptr}, {w.gu, 0, nullptr, nullptr}, {w.down, 0, nullptr, nullptr},
                          {m->out, 0, nullptr, nullptr}};
  size_t pf = 0;
  int tk = 0;
  for (int i = -1; i < 4; ++i) {
    const SegSpec* ss = i < 0 ? qkv : &one[i];
    const int nseg = i < 0 ? 3 : 1, tiles = tmm_tiles(ss, nseg);
    pf = std::max(pf, tmm_part_floats(tiles, tmm_split(tiles, ss[0].m->C / 256, m->nsm), MM_MAXM));
    tk = std::max(tk, tiles);
  }
  m->tpart_floats = pf;
  m->tticket_n = tk;
  m->tpart = dalloc<float>(m, std::max<size_t>(pf, 1), ok);
  m->tticket = dalloc<int>(m, (size_t)tk, ok);
  if (!ok) return set_err(KQ_ERR_MEMORY, "batched verify buffers");
  return KQ_OK;
}

static bool batch_supported(const kq_model* m) {
  return m->ffn_l % 64 == 0 && (m->nh_l * m->c.head_dim) % 64 == 0;
}

// xscale: the per-token scales of the packed input xp (k_bnorm / k_xpack_tok), or null; xsum: its
// sub-block sums (they enable the exact form for Q4_K row tiles), or null.
static int launch_tmm(kq_model* m, const SegSpec* ss, int nseg, const __half* xp, const float* xscale,
                      const float* xsum, int out_ld, const BatchParams& B) {
  prof_mark(m, PC_GEMM);
  TmmParams P;
  tmm_fill(ss, nseg, B.M, m->device, P);
  P.xp = xp;
  P.xscale = xscale;
  P.xsum = tmm_exact_ok() ? xsum : nullptr;
  P.B = B;
  P.out_ld = out_ld;
  P.cos_t = m->cos_t;
  P.sin_t = m->sin_t;
  P.hd = m->c.head_dim;
  P.ctx = m->c.ctx;
  P.nkv = m->nkv_l;
  P.part = m->tpart;
  P.ticket = m->tticket;
  P.err = m->err;
  if (tmm_part_floats(P.ntiles, P.nsplit, P.Npad) > m->tpart_floats || P.ntiles > m->tticket_n)
    return set_err(KQ_ERR_BACKEND, "GEMM scratch too small");
  CU(tmm_launch(P, m->stream, true));
  return KQ_OK;
}

static int launch_bnorm(kq_model* m, int M, bool embed, const float* gamma, bool add) {
  prof_mark(m, PC_OTHER);
  BNormParams P;
  std::memset(&P, 0, sizeof(P));
  P.M = M; P.D = m->c.dim; P.tok = m->btok;
  if (embed) P.emb = m->emb->view();
  P.h = m->bh; P.y = add ? m->by : nullptr; P.gamma = gamma; P.eps = m->c.eps;
  P.xp = m->bxd; P.xscale = m->bxs_n; P.xsum = m->bxd_sum; P.Npad = (M + 15) & ~15;
  P.vocab = m->c.vocab; P.err = m->err;
  CU(launch_pdl(k_bnorm, dim3((unsigned)M), dim3(BN_THREADS), 0, m->stream, P));
  return KQ_OK;
}

// The MLP of a batched pass after its norm (bxd): gate/up GEMM with the SwiGLU epilogue (fp32
// rows in bmf), the per-token range-scaled packing of those rows (k_xpack_tok), the down GEMM
// into y (M x dim).
static int launch_mlp(kq_model* m, LayerW& w, float* y, const BatchParams& B) {
  const int M = B.M, Npad = (M + 15) & ~15;
  SegSpec sg[1] = {{w.gu, EPI_SWIGLU, m->bmf, nullptr}};
  int rc = launch_tmm(m, sg, 1, m->bxd, m->bxs_n, m->bxd_sum, m->ffn_l, B);
  if (rc) return rc;
  prof_mark(m, PC_GEMM);
  const XPackParams X = {m->bmf, m->ffn_l, m->ffn_l, Npad, m->bxf, m->bxs_f, m->bxf_sum};
  CU(launch_pdl(k_xpack_tok, dim3((unsigned)M), dim3(XP_THREADS), 0, m->stream, X));
  SegSpec sd[1] = {{w.down, EPI_F32, y, nullptr}};
  return launch_tmm(m, sd, 1, m->bxf, m->bxs_f, m->bxf_sum, m->c.dim, B);
}

static int launch_battn(kq_model* m, const __half* kc, const __half* vc, int npos, const BatchParams& B) {
  prof_mark(m, PC_ATTN);
  const kq_config& c = m->c;
  const int G = c.n_heads / c.n_kv_heads, M = B.M;
  const int rowgroups = (M * G + BA_ROWS - 1) / BA_ROWS, nblocks = (npos + BA_KB - 1) / BA_KB;
  const int base = m->nkv_l * rowgroups;
  int want = std::max(1, (2 * m->nsm + base - 1) / base);
  want = std::min(want, std::min(nblocks, m->b_nsplit));
  BAttnParams P;
  P.q = m->bq; P.kc = kc; P.vc = vc; P.out_xp = m->bxa; P.Npad = (M + 15) & ~15; P.B = B;
  P.n_kv = m->nkv_l; P.ctx = c.ctx; P.npos = npos;
  P.scale = (float)(1.0 / std::sqrt((double)c.head_dim));
  P.nblk = (nblocks + want - 1) / want;
  P.nsplit = (nblocks + P.nblk - 1) / P.nblk;
  P.part = m->bpart; P.ticket = m->bticket;
  const dim3 grid((unsigned)m->nkv_l, (unsigned)rowgroups, (unsigned)P.nsplit), blk(BA_WARPS * 32);
  cudaError_t e;
  if (G == 1) e = launch_pdl(k_battn<1>, grid, blk, BA_SMEM, m->stream, P);
  else if (G == 2) e = launch_pdl(k_battn<2>, grid, blk, BA_SMEM, m->stream, P);
  else if (G == 4) e = launch_pdl(k_battn<4>, grid, blk, BA_SMEM, m->stream, P);
  else e = launch_pdl(k_battn<8>, grid, blk, BA_SMEM, m->stream, P);
  CU(e);
  return KQ_OK;
}

// One batched pass over nodes [b0, b1) of a verified tree (their ancestors are in this or an
// earlier pass): node i's K/V to slot pos + i, rotary position pos + depth[i], attention to the
// slots below pos and its ancestors (anc, bits relative to pos). With `head`: logits to vlogits
// rows b0.., argmax ids to out_ids[b0..]; without (prefill): the K/V cache only.
static int verify_pass(kq_model* m, const int32_t* tokens, int b0, int b1, int pos, const int* depth,
                       const unsigned long long (*anc)[2], bool head, int seq) {
  const kq_config& c = m->c;
  const int M = b1 - b0;
  kq_model::MetaSlot* ms = nullptr;
  int rc = meta_acquire(m, &ms);
  if (rc) return rc;
  for (int i = 0; i < M; ++i) {
    ms->tok[i] = tokens[b0 + i];
    ms->slot[i] = pos + b0 + i;
    ms->rpos[i] = pos + depth[b0 + i];
    ms->mask[2 * i] = anc[b0 + i][0];
    ms->mask[2 * i + 1] = anc[b0 + i][1];
  }
  cudaStream_t s = m->stream;
  CU(cudaMemcpyAsync(m->btok, ms->tok, M * sizeof(int), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->bslot, ms->slot, M * sizeof(int), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->brpos, ms->rpos, M * sizeof(int), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->bmask, ms->mask, 2 * M * sizeof(unsigned long long), cudaMemcpyHostToDevice, s));
  if ((rc = meta_release(m))) return rc;
  BatchParams B;
  B.M = M; B.slot = m->bslot; B.rpos = m->brpos; B.mask = m->bmask; B.tree_base = pos; B.seq = nullptr;
  const size_t sstride = (size_t)m->nkv_l * c.ctx * c.head_dim;   // one sequence of the batched-decode caches
  const int QD = m->nh_l * c.head_dim;
  for (int l = 0; l < c.n_layers; ++l) {
    LayerW& w = m->L[l];
    if ((rc = launch_bnorm(m, M, l == 0, w.attn_norm, l > 0))) return rc;
    __half* kc = seq < 0 ? w.kc : w.bkc + (size_t)seq * sstride;
    __half* vc = seq < 0 ? w.vc : w.bvc + (size_t)seq * sstride;
    SegSpec qkv[3] = {{w.q, EPI_ROPE_Q, m->bq, nullptr}, {w.k, EPI_ROPE_K, nullptr, kc}, {w.v, EPI_V, nullptr, vc}};
    if ((rc = launch_tmm(m, qkv, 3, m->bxd, m->bxs_n, m->bxd_sum, QD, B))) return rc;
    if ((rc = launch_battn(m, kc, vc, pos + b1, B))) return rc;
    SegSpec so[1] = {{w.o, EPI_F32, m->by, nullptr}};
    if ((rc = launch_tmm(m, so, 1, m->bxa, nullptr, nullptr, c.dim, B))) return rc;   // attention output: |x| <= max|V|
    if ((rc = tp_allreduce(m, m->by, (size_t)M * c.dim))) return rc;   // row-split o: sum the partials
    if ((rc = launch_bnorm(m, M, false, w.ffn_norm, true))) return rc;
    if ((rc = launch_mlp(m, w, m->by, B))) return rc;
    if ((rc = tp_allreduce(m, m->by, (size_t)M * c.dim))) return rc;   // row-split down
  }
  if (!head) return KQ_OK;
  return head_argmax(m, M, B, m->out_ids + b0, (size_t)b0);
}

// Final norm, output head and per-token greedy id of a batched pass's M tokens (logits to vlogits
// rows row0.., ids to out_ids); a tensor-parallel rank gathers the ranks' (value, id) pairs.
static int head_argmax(kq_model* m, int M, const BatchParams& B, int* out_ids, size_t row0) {
  int rc;
  cudaStream_t s = m->stream;
  if ((rc = launch_bnorm(m, M, false, m->out_norm, true))) return rc;
  const size_t V = (size_t)m->vocab_l;   // this rank's vocabulary slice
  SegSpec sh[1] = {{m->out, EPI_F32, m->vlogits + row0 * V, nullptr}};
  if ((rc = launch_tmm(m, sh, 1, m->bxd, m->bxs_n, m->bxd_sum, (int)V, B))) return rc;
  prof_mark(m, PC_OTHER);
  if (m->tp_world == 1) {
    k_argmax_rows<<<M, 256, 0, s>>>(m->vlogits + row0 * V, (int)V, out_ids);
    CU(cudaGetLastError());
    return KQ_OK;
  }
  // vocabulary-split head: each rank's (best value, global id) per token, gathered, then the
  // best over ranks (rank order = id order, so ties keep the lowest id)
  const int W = m->tp_world;
  float* sv = m->tp_val + (size_t)W * MM_MAXM;
  int* si = m->tp_idx + (size_t)W * MM_MAXM;
  k_argmax_rows_vi<<<M, 256, 0, s>>>(m->vlogits + row0 * V, (int)V, m->tp_rank * (int)V, sv, si);
  CU(cudaGetLastError());
  if ((rc = tp_alive(m)) ||
      (rc = nccl_wait(m, nccl().AllGather(sv, m->tp_val, (size_t)MM_MAXM, ncclFloat32, m->comm, s), "ncclAllGather")) ||
      (rc = nccl_wait(m, nccl().AllGather(si, m->tp_idx, (size_t)MM_MAXM, ncclInt32, m->comm, s), "ncclAllGather")))
    return rc;
  k_pick_rows<<<(M + 127) / 128, 128, 0, s>>>(m->tp_val, m->tp_idx, W, MM_MAXM, M, out_ids);
  CU(cudaGetLastError());
  return KQ_OK;
}

extern "C" int kq_verify(kq_model* m, const int32_t* tokens, const int32_t* parents, int n, int pos, float* logits,
                         int32_t* best) {
  int rc = model_check(m);
  if (rc) return rc;
  int depth[KQ_MAX_TREE];
  unsigned long long anc[KQ_MAX_TREE][2];
  if ((rc = tree_check(parents, n, depth, anc))) return rc;
  if (!tokens || pos < 0) return set_err(KQ_ERR_ARG, "bad verify arguments");
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= m->c.vocab) return set_err(KQ_ERR_ARG, "Invalid token in the draft tree");
  if (pos + n > m->c.ctx) return set_err(KQ_ERR_OVERFLOW, "draft tree runs past the context");
  if (m->tp_world > 1 && logits) return set_err(KQ_ERR_ARG, "a tensor-parallel shard holds a vocabulary slice: request best ids only");
  if ((m->tp_world == 1 && (rc = ensure_graphs(m))) || (rc = verify_buffers(m))) return rc;
  const size_t V = (size_t)m->vocab_l;
  const bool batched = m->tp_world > 1 || (!m->verify_seq && batch_supported(m));
  if (batched) {
    if ((rc = batch_buffers(m))) return rc;
    for (int b0 = 0; b0 < n; b0 += MM_MAXM)
      if ((rc = verify_pass(m, tokens, b0, std::min(n, b0 + MM_MAXM), pos, depth, anc))) return rc;
  }
  for (int i = 0; i < n && !batched; ++i) {
    DecodeState& st = m->vstates[i];
    std::memset(&st, 0, sizeof(st));
    st.tok = tokens[i];
    st.pos = pos + i;            // K/V slot
    st.next_tok = -1;
    st.steps = i;                // the head's argmax lands in out_ids[i]
    st.rpos = pos + depth[i];    // rotary position
    st.tree_base = pos;
    st.mask[0] = anc[i][0];
    st.mask[1] = anc[i][1];
    CU(cudaMemcpyAsync(m->st, &st, sizeof(DecodeState), cudaMemcpyHostToDevice, m->stream));
    if (m->persist) {
      if ((rc = launch_persistent(m, true))) return rc;
    } else {
      CU(cudaGraphLaunch(m->g_step, m->stream));
    }
    CU(cudaMemcpyAsync(m->vlogits + i * V, m->logits, V * sizeof(float), cudaMemcpyDeviceToDevice, m->stream));
  }
  prof_mark(m, PC_END);
  if ((rc = tp_sync(m))) return rc;   // the results are read once the stream drained (bounded for TP)
  prof_flush(m);
  if (best) CU(cudaMemcpyAsync(best, m->out_ids, (size_t)n * sizeof(int32_t), cudaMemcpyDeviceToHost, m->stream));
  if (logits) CU(cudaMemcpyAsync(logits, m->vlogits, (size_t)n * V * sizeof(float), cudaMemcpyDeviceToHost, m->stream));
  if (best || logits) CU(cudaStreamSynchronize(m->stream));
  m->vn = n;
  return check_dev_err(m);
}

// draft_logits: host rows copied in (kq_accept), or null with `resident`: the rows are already in
// the model's device buffer (kq_accept_resident; a drafter on the GPU writes there, see
// kq_draft_logits).
static int accept_impl(kq_model* m, const int32_t* tokens, const int32_t* parents, int n, const float* draft_logits,
                       bool resident, float temperature, const float* u_acc, const float* u_fin, int32_t* path,
                       int32_t* out, int32_t* path_len) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "kq_accept"))) return rc;
  if (resident) draft_logits = m->ag;
  int depth[KQ_MAX_TREE];
  unsigned long long anc[KQ_MAX_TREE][2];
  if ((rc = tree_check(parents, n, depth, anc))) return rc;
  if (!tokens || !path || !out || !(temperature >= 0.0f)) return set_err(KQ_ERR_ARG, "bad accept arguments");
  if (temperature > 0.0f && (!draft_logits || !u_acc || !u_fin)) return set_err(KQ_ERR_ARG, "stochastic acceptance needs draft logits and uniforms");
  if (!m->vlogits || m->vn != n) return set_err(KQ_ERR_ARG, "kq_accept needs the logits of a kq_verify over the same tree");
  if (m->c.vocab > ACC_BLK * ACC_MAX_BLOCKS) return set_err(KQ_ERR_ARG, "vocabulary too large for the acceptance kernel");
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= m->c.vocab) return set_err(KQ_ERR_ARG, "Invalid token in the draft tree");
  const size_t V = (size_t)m->c.vocab;
  cudaStream_t s = m->stream;
  CU(cudaMemcpyAsync(m->atok, tokens, n * sizeof(int32_t), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->apar, parents, n * sizeof(int32_t), cudaMemcpyHostToDevice, s));
  AcceptParams A;
  std::memset(&A, 0, sizeof(A));
  A.tau = temperature > 0.0f ? 1.0f / temperature : 0.0f;
  if (A.tau > 0.0f) {
    if (!resident) CU(cudaMemcpyAsync(m->ag, draft_logits, n * V * sizeof(float), cudaMemcpyHostToDevice, s));
    CU(cudaMemcpyAsync(m->auacc, u_acc, n * sizeof(float), cudaMemcpyHostToDevice, s));
    CU(cudaMemcpyAsync(m->aufin, u_fin, n * sizeof(float), cudaMemcpyHostToDevice, s));
  }
  A.z = m->vlogits; A.g = m->ag; A.tokens = m->atok; A.parents = m->apar; A.u_acc = m->auacc; A.u_fin = m->aufin;
  A.n = n; A.V = (int)V; A.p = m->ap; A.q = m->aq; A.path = m->apath; A.out = m->aout; A.count = m->acnt;
  A.err = m->err;
  // the multi-CTA form (a cooperative grid of ceil(blocks / 2) CTAs) unless KQ_ACCEPT_GRID=0 asks
  // for the one-CTA kernel (comparison) or the grid cannot be co-resident
  const int nbk = (int)((V + ACC_BLK - 1) / ACC_BLK), nc = (nbk + 1) / 2;
  const char* eg = std::getenv("KQ_ACCEPT_GRID");
  int coop = 0, per_sm = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device);
  if (coop) CU(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_accept_grid, ACC_THREADS, 0));
  if (!(eg && std::atoi(eg) == 0) && coop && nc <= per_sm * m->nsm) {
    CU(cudaMemsetAsync(&m->agrid->bar, 0, sizeof(unsigned), s));
    CU(cudaMemsetAsync(&m->agrid->pick, 0xFF, sizeof(unsigned) + sizeof(int), s));   // pick, hi
    AccGridScratch* G = m->agrid;
    void* args[] = {(void*)&A, (void*)&G};
    CU(cudaLaunchCooperativeKernel((const void*)k_accept_grid, dim3((unsigned)nc), dim3(ACC_THREADS), args, 0, s));
  } else {
    k_accept<<<1, ACC_THREADS, 0, s>>>(A);
  }
  CU(cudaGetLastError());
  int cnt[2] = {0, 0};
  CU(cudaMemcpyAsync(cnt, m->acnt, sizeof(cnt), cudaMemcpyDeviceToHost, s));
  CU(cudaStreamSynchronize(s));
  if (cnt[0] < 1 || cnt[0] > n + 1 || cnt[1] < 1 || cnt[1] > n) {
    // a grid-barrier wait of the multi-CTA form that gave up is reported (and the error word
    // cleared) here rather than by the next call
    const int rc2 = check_dev_err(m);
    return rc2 ? rc2 : set_err(KQ_ERR_BACKEND, "acceptance kernel failed");
  }
  CU(cudaMemcpy(out, m->aout, cnt[0] * sizeof(int32_t), cudaMemcpyDeviceToHost));
  CU(cudaMemcpy(path, m->apath, cnt[1] * sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (path_len) *path_len = cnt[1];
  return cnt[0];
}

extern "C" int kq_accept(kq_model* m, const int32_t* tokens, const int32_t* parents, int n, const float* draft_logits,
                         float temperature, const float* u_acc, const float* u_fin, int32_t* path, int32_t* out,
                         int32_t* path_len) {
  return accept_impl(m, tokens, parents, n, draft_logits, false, temperature, u_acc, u_fin, path, out, path_len);
}
extern "C" int kq_accept_resident(kq_model* m, const int32_t* tokens, const int32_t* parents, int n, float temperature,
                                  const float* u_acc, const float* u_fin, int32_t* path, int32_t* out, int32_t* path_len) {
  return accept_impl(m, tokens, parents, n, nullptr, true, temperature, u_acc, u_fin, path, out, path_len);
}
extern "C" int kq_draft_logits(kq_model* m, float** dev, int* ld) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "kq_draft_logits")) || (rc = verify_buffers(m))) return rc;
  if (dev) *dev = m->ag;
  if (ld) *ld = m->c.vocab;
  return KQ_OK;
}
extern "C" int kq_draft_upload(kq_model* m, const float* host, int n) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "kq_draft_upload")) || (rc = verify_buffers(m))) return rc;
  if (!host || n < 1 || n > KQ_MAX_TREE) return set_err(KQ_ERR_ARG, "bad draft logits");
  CU(cudaMemcpy(m->ag, host, (size_t)n * m->c.vocab * sizeof(float), cudaMemcpyHostToDevice));
  return KQ_OK;
}

// ------------------------------------------------------------------------------ batched decode
// Many sequences at once (config-4 decode): each has its own K/V cache [n_kv][ctx][hd] per layer;
// a step takes one token per sequence through the batched pass (the weights stream once for all
// of them) with attention over each token's own cache. Whole and tensor-parallel models alike.
extern "C" int kq_batch_caches(kq_model* m, int n_seq) {
  int rc = model_check(m);
  if (rc) return rc;
  if (n_seq < 1) return set_err(KQ_ERR_ARG, "n_seq must be positive");
  if (m->n_seq) return m->n_seq == n_seq ? KQ_OK : set_err(KQ_ERR_ARG, "the batched-decode caches are already allocated");
  const kq_config& c = m->c;
  const size_t per = (size_t)n_seq * m->nkv_l * c.ctx * c.head_dim;
  bool ok = true;
  for (auto& w : m->L) {
    w.bkc = dalloc<__half>(m, per, ok);
    w.bvc = dalloc<__half>(m, per, ok);
    if (!ok) break;
  }
  const int G = c.n_heads / c.n_kv_heads;
  if (ok) {
    m->bseq = dalloc<int>(m, MM_MAXM, ok);
    m->bposv = dalloc<int>(m, MM_MAXM, ok);
    m->dpart = dalloc<float>(m, (size_t)MM_MAXM * m->nkv_l * DA_MAX_SPLIT * G * (c.head_dim + 4), ok);
  }
  if (!ok) return set_err(KQ_ERR_MEMORY, "batched-decode caches");
  m->n_seq = n_seq;
  return KQ_OK;
}

// Prefill of sequence `seq`'s cache (chunks of up to MM_MAXM tokens, as kq_feed_batch).
extern "C" int kq_batch_feed(kq_model* m, int seq, const int32_t* toks, int n, int pos) {
  int rc = model_check(m);
  if (rc) return rc;
  if (seq < 0 || seq >= m->n_seq) return set_err(KQ_ERR_ARG, "sequence out of range (kq_batch_caches first)");
  if (!toks || n < 1 || pos < 0) return set_err(KQ_ERR_ARG, "bad token batch");
  for (int i = 0; i < n; ++i)
    if (toks[i] < 0 || toks[i] >= m->c.vocab) return set_err(KQ_ERR_ARG, "Invalid token");
  if (pos + n > m->c.ctx) return set_err(KQ_ERR_OVERFLOW, "prompt runs past the context");
  if (!batch_supported(m)) return set_err(KQ_ERR_ARG, "configuration not covered by the batched pass");
  if ((rc = verify_buffers(m)) || (rc = batch_buffers(m))) return rc;
  static const ChainMasks chain;
  for (int c0 = 0; c0 < n; c0 += MM_MAXM)
    if ((rc = verify_pass(m, toks + c0, 0, std::min(MM_MAXM, n - c0), pos + c0, chain.depth, chain.anc, false, seq)))
      return rc;
  if ((rc = tp_sync(m))) return rc;
  return check_dev_err(m);
}

// One decode step for n sequences: token toks[i] at position pos[i] of sequence seqs[i] (distinct
// sequences). Writes the greedy ids to out[i] and the K/V rows to the sequences' caches.
extern "C" int kq_batch_step(kq_model* m, const int32_t* seqs, const int32_t* toks, const int32_t* pos, int n,
                             int32_t* out) {
  int rc = model_check(m);
  if (rc) return rc;
  if (!seqs || !toks || !pos || !out || n < 1 || n > MM_MAXM) return set_err(KQ_ERR_ARG, "bad batched step arguments");
  const kq_config& c = m->c;
  int maxpos = 0;
  for (int i = 0; i < n; ++i) {
    if (seqs[i] < 0 || seqs[i] >= m->n_seq) return set_err(KQ_ERR_ARG, "sequence out of range (kq_batch_caches first)");
    if (toks[i] < 0 || toks[i] >= c.vocab || pos[i] < 0) return set_err(KQ_ERR_ARG, "Invalid token or position");
    if (pos[i] >= c.ctx) return set_err(KQ_ERR_OVERFLOW, "position past the context");
    for (int j = 0; j < i; ++j)
      if (seqs[j] == seqs[i]) return set_err(KQ_ERR_ARG, "one token per sequence in a batched step");
    maxpos = std::max(maxpos, pos[i]);
  }
  if (!batch_supported(m)) return set_err(KQ_ERR_ARG, "configuration not covered by the batched pass");
  if ((rc = verify_buffers(m)) || (rc = batch_buffers(m))) return rc;
  cudaStream_t s = m->stream;
  const int M = n;
  kq_model::MetaSlot* ms = nullptr;
  if ((rc = meta_acquire(m, &ms))) return rc;
  std::memcpy(ms->tok, toks, M * sizeof(int));
  std::memcpy(ms->slot, pos, M * sizeof(int));
  std::memcpy(ms->seq, seqs, M * sizeof(int));
  CU(cudaMemcpyAsync(m->btok, ms->tok, M * sizeof(int), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->bslot, ms->slot, M * sizeof(int), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->brpos, ms->slot, M * sizeof(int), cudaMemcpyHostToDevice, s));
  CU(cudaMemcpyAsync(m->bseq, ms->seq, M * sizeof(int), cudaMemcpyHostToDevice, s));
  if ((rc = meta_release(m))) return rc;
  BatchParams B;
  std::memset(&B, 0, sizeof(B));
  B.M = M; B.slot = m->bslot; B.rpos = m->brpos; B.seq = m->bseq;
  const int G = c.n_heads / c.n_kv_heads, QD = m->nh_l * c.head_dim;
  DAttnParams D;
  std::memset(&D, 0, sizeof(D));
  D.q = m->bq; D.seq = m->bseq; D.pos = m->bslot; D.n_kv = m->nkv_l; D.ctx = c.ctx;
  D.scale = (float)(1.0 / std::sqrt((double)c.head_dim));
  D.part = m->dpart; D.out_xp = m->bxa; D.Npad = (M + 15) & ~15;
  // splits: about six one-warp CTAs per SM, at least two 32-key blocks each
  D.nsplit = std::max(1, std::min(DA_MAX_SPLIT, std::min((6 * m->nsm + M * m->nkv_l - 1) / (M * m->nkv_l), (maxpos + 64) / 64)));
  for (int l = 0; l < c.n_layers; ++l) {
    LayerW& w = m->L[l];
    if ((rc = launch_bnorm(m, M, l == 0, w.attn_norm, l > 0))) return rc;
    SegSpec qkv[3] = {{w.q, EPI_ROPE_Q, m->bq, nullptr}, {w.k, EPI_ROPE_K, nullptr, w.bkc}, {w.v, EPI_V, nullptr, w.bvc}};
    if ((rc = launch_tmm(m, qkv, 3, m->bxd, m->bxs_n, m->bxd_sum, QD, B))) return rc;
    D.kc = w.bkc;
    D.vc = w.bvc;
    prof_mark(m, PC_ATTN);
    cudaError_t e = G == 1 ? launch_dattn_t<1>(D, M, m->nkv_l, s) : G == 2 ? launch_dattn_t<2>(D, M, m->nkv_l, s)
                  : G == 4 ? launch_dattn_t<4>(D, M, m->nkv_l, s) : launch_dattn_t<8>(D, M, m->nkv_l, s);
    CU(e);
    SegSpec so[1] = {{w.o, EPI_F32, m->by, nullptr}};
    if ((rc = launch_tmm(m, so, 1, m->bxa, nullptr, nullptr, c.dim, B))) return rc;   // attention output: |x| <= max|V|
    if ((rc = tp_allreduce(m, m->by, (size_t)M * c.dim))) return rc;
    if ((rc = launch_bnorm(m, M, false, w.ffn_norm, true))) return rc;
    if ((rc = launch_mlp(m, w, m->by, B))) return rc;
    if ((rc = tp_allreduce(m, m->by, (size_t)M * c.dim))) return rc;
  }
  if ((rc = head_argmax(m, M, B, m->out_ids))) return rc;
  prof_mark(m, PC_END);
  if ((rc = tp_sync(m))) return rc;
  prof_flush(m);
  CU(cudaMemcpy(out, m->out_ids, M * sizeof(int32_t), cudaMemcpyDeviceToHost));
  return check_dev_err(m);
}

extern "C" int kq_commit(kq_model* m, const int32_t* path, int k, int pos) {
  int rc = model_check(m);
  if (rc) return rc;
  if (!path || k < 0 || k >= KQ_MAX_TREE || pos < 0 || path[0] != 0) return set_err(KQ_ERR_ARG, "bad commit arguments");
  for (int j = 1; j <= k; ++j)
    if (path[j] <= path[j - 1] || path[j] >= KQ_MAX_TREE) return set_err(KQ_ERR_ARG, "bad commit path (node ids must increase)");
  if (pos + (k ? path[k] : 0) >= m->c.ctx) return set_err(KQ_ERR_OVERFLOW, "commit path runs past the context");
  if (k == 0) return KQ_OK;
  if ((rc = verify_buffers(m))) return rc;
  CU(cudaMemcpyAsync(m->apath, path, (size_t)(k + 1) * sizeof(int32_t), cudaMemcpyHostToDevice, m->stream));
  CommitParams C;
  C.caches = m->caches; C.path = m->apath; C.k = k; C.pos = pos;
  C.n_kv = m->nkv_l; C.ctx = m->c.ctx; C.hd = m->c.head_dim;
  k_commit<<<2 * m->c.n_layers, 256, 0, m->stream>>>(C);
  CU(cudaGetLastError());
  CU(cudaStreamSynchronize(m->stream));
  return KQ_OK;
}

#ifdef KQ_TRACE
// Trace builds only (not part of include/kq.h): copy the phase-trace buffer to the host.
extern "C" int kq_trace_read(unsigned long long* out, size_t n) {
  const size_t total = (size_t)KQ_TRACE_LAUNCHES * KQ_TRACE_CTAS * KQ_TRACE_POINTS;
  if (n > total) n = total;
  CU(cudaMemcpyFromSymbol(out, g_kq_trace, n * sizeof(unsigned long long)));
  return KQ_OK;
}
extern "C" int kq_trace_clear(void) {
  static unsigned long long zero[KQ_TRACE_CTAS * KQ_TRACE_POINTS];
  for (int l = 0; l < KQ_TRACE_LAUNCHES; ++l)
    CU(cudaMemcpyToSymbol(g_kq_trace, zero, sizeof(zero), (size_t)l * sizeof(zero)));
  return KQ_OK;
}
#endif

// ------------------------------------------------------------------------------ matrix hooks
extern "C" kq_qmat* kq_qmat_create(int type, int rows, int cols, int device) { return qmat_alloc(type, rows, cols, device); }
extern "C" void kq_qmat_free(kq_qmat* a) {
  if (!a) return;
  cudaSetDevice(a->device);
  cudaFree(a->buf);
  cudaFree(a->tvbuf);
  cudaFree(a->tv_part);
  cudaFree(a->tv_ticket);
  delete a;
}
extern "C" size_t kq_qmat_bytes(const kq_qmat* a) { return a ? a->bytes : 0; }

extern "C" int kq_qmat_upload(kq_qmat* a, const void* bytes_host, size_t bytes) {
  if (!a || !bytes_host) return set_err(KQ_ERR_ARG, "null argument");
  CU(cudaSetDevice(a->device));
  return qmat_upload_mapped(a, bytes_host, bytes, a->R, RM_IDENT, 0, 0);
}

extern "C" int kq_qmat_fill_synthetic(kq_qmat* a, uint64_t seed, uint64_t stream) {
  if (!a) return set_err(KQ_ERR_ARG, "null matrix");
  CU(cudaSetDevice(a->device));
  int rc = qmat_write(a, a->R, nullptr, gen_base(seed, stream), RM_IDENT, 0, 0);
  if (rc) return rc;
  CU(cudaDeviceSynchronize());
  return KQ_OK;
}

extern "C" int kq_qmat_dequant(kq_qmat* a, int row, int nrows, float* out) {
  if (!a || !out || row < 0 || nrows < 1 || row + nrows > a->R) return set_err(KQ_ERR_ARG, "bad dequant request");
  CU(cudaSetDevice(a->device));
  float* d = nullptr;
  const size_t n = (size_t)nrows * a->C;
  CU(cudaMalloc(&d, n * 4));
  k_qmat_dequant<<<(unsigned)((n + 255) / 256), 256>>>(a->view(), row, nrows, d);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaMemcpy(out, d, n * 4, cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return set_err(KQ_ERR_BACKEND, std::string("dequant: ") + cudaGetErrorString(e));
  return KQ_OK;
}

// One matrix-vector product y = W x: the tensor-core GEMV where it covers the shape, else k_gemv.
struct MatvecLaunch {
  GemvParams p;
  GemvPlan pl;
  bool tmv = false;
  TmvParams t;
  dim3 grid;
};

static int qmat_gemv_params(kq_qmat* a, const float* x_dev, float* y_dev, MatvecLaunch& L) {
  int rc = dev_init(a->device);
  if (rc) return rc;
  SegSpec ss[1] = {{a, EPI_F32, y_dev, nullptr}};
  if ((rc = fill_gemv(ss, 1, false, g_dev[a->device].nsm, L.p, L.pl))) return rc;
  L.p.xmode = XS_PLAIN;
  L.p.x = x_dev;
  L.p.err = g_dev[a->device].err;
  const DevCtx& D = g_dev[a->device];
  if (D.tmv_smem > 0 && !a->tv_part) {
    if (cudaMalloc(&a->tv_part, (size_t)D.nsm * 2 * TV_ROWS * 4) != cudaSuccess ||
        cudaMalloc(&a->tv_ticket, (size_t)TV_MAX_TILES * 4) != cudaSuccess ||
        cudaMemset(a->tv_ticket, 0, (size_t)TV_MAX_TILES * 4) != cudaSuccess)
      return set_err(KQ_ERR_MEMORY, "matvec scratch");
  }
  L.tmv = !L.pl.mma && tmv_plan(L.p, D.nsm, D.tmv_smem, a->tv_part, a->tv_ticket, L.t, L.grid);
  return KQ_OK;
}
static cudaError_t matvec_launch(const MatvecLaunch& L, cudaStream_t s, bool pdl) {
  if (L.tmv) return launch_pdl(k_tmv, L.grid, dim3(TV_THREADS), (size_t)L.t.smem, s, L.t);
  return launch_gemv(L.p, L.pl, s, pdl);
}

extern "C" int kq_qmat_matvec_dev(kq_qmat* a, const float* x_dev, float* y_dev, void* stream) {
  if (!a || !x_dev || !y_dev) return set_err(KQ_ERR_ARG, "null argument");
  CU(cudaSetDevice(a->device));
  MatvecLaunch L;
  int rc = qmat_gemv_params(a, x_dev, y_dev, L);
  if (rc) return rc;
  CU(matvec_launch(L, (cudaStream_t)stream, false));
  return KQ_OK;
}

static int dev_err_check(int device) {
  int e = 0;
  CU(cudaMemcpy(&e, g_dev[device].err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    cudaMemset(g_dev[device].err, 0, sizeof(int));
    return set_err(KQ_ERR_TIMEOUT, "a bounded device wait gave up");
  }
  return KQ_OK;
}

extern "C" int kq_qmat_matvec(kq_qmat* a, const float* x, float* y) {
  if (!a || !x || !y) return set_err(KQ_ERR_ARG, "null argument");
  CU(cudaSetDevice(a->device));
  float *xd = nullptr, *yd = nullptr;
  CU(cudaMalloc(&xd, (size_t)a->C * 4));
  if (cudaMalloc(&yd, (size_t)a->R * 4) != cudaSuccess) { cudaFree(xd); return set_err(KQ_ERR_MEMORY, "matvec buffers"); }
  int rc = KQ_OK;
  if (cudaMemcpy(xd, x, (size_t)a->C * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "matvec upload");
  if (!rc) rc = kq_qmat_matvec_dev(a, xd, yd, nullptr);
  if (!rc && cudaMemcpy(y, yd, (size_t)a->R * 4, cudaMemcpyDeviceToHost) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "matvec download");
  cudaFree(xd);
  cudaFree(yd);
  if (!rc) rc = dev_err_check(a->device);
  return rc;
}

// M = 1: the decode GEMV; M >= 2: the tensor-core GEMM of the batched passes (split-precision
// fp16 operands, fp32 accumulation).
extern "C" int kq_qmat_matmul(kq_qmat* a, const float* x, int M, float* y) {
  if (!a || !x || !y || M < 1 || M > 64) return set_err(KQ_ERR_ARG, "bad matmul arguments");
  if (M == 1) return kq_qmat_matvec(a, x, y);
  int rc = dev_init(a->device);
  if (rc) return rc;
  CU(cudaSetDevice(a->device));
  const SegSpec ss[1] = {{a, EPI_F32, nullptr, nullptr}};
  TmmParams P;
  tmm_fill(ss, 1, M, a->device, P);
  const size_t pf = tmm_part_floats(P.ntiles, P.nsplit, P.Npad);
  float *xd = nullptr, *yd = nullptr, *part = nullptr, *xs = nullptr, *xsum = nullptr;
  __half* xp = nullptr;
  int* ticket = nullptr;
  const bool sums = a->C % 256 == 0 && tmm_exact_ok();
  bool ok = cudaMalloc(&xd, (size_t)M * a->C * 4) == cudaSuccess;
  ok = ok && cudaMalloc(&xs, (size_t)M * 4) == cudaSuccess;
  ok = ok && (!sums || cudaMalloc(&xsum, (size_t)P.Npad * (a->C / 32) * 4) == cudaSuccess);
  ok = ok && cudaMalloc(&yd, (size_t)M * a->R * 4) == cudaSuccess;
  ok = ok && cudaMalloc(&xp, xp_halves(P.Npad, a->C) * 2) == cudaSuccess;
  ok = ok && cudaMalloc(&part, std::max<size_t>(pf, 1) * 4) == cudaSuccess;
  ok = ok && cudaMalloc(&ticket, (size_t)P.ntiles * 4) == cudaSuccess;
  if (!ok) rc = set_err(KQ_ERR_MEMORY, "matmul buffers");
  if (!rc && (cudaMemset(ticket, 0, (size_t)P.ntiles * 4) != cudaSuccess ||
              cudaMemset(xp, 0, xp_halves(P.Npad, a->C) * 2) != cudaSuccess ||
              cudaMemcpy(xd, x, (size_t)M * a->C * 4, cudaMemcpyHostToDevice) != cudaSuccess))
    rc = set_err(KQ_ERR_BACKEND, "matmul upload");
  if (!rc) {
    const XPackParams X = {xd, a->C, a->C, P.Npad, xp, xs, xsum};
    k_xpack_tok<<<(unsigned)M, XP_THREADS>>>(X);
    P.xp = xp;
    P.xscale = xs;
    P.xsum = xsum;
    P.seg[0].out_f = yd;
    P.out_ld = a->R;
    P.part = part;
    P.ticket = ticket;
    P.err = g_dev[a->device].err;
    if (cudaGetLastError() != cudaSuccess || tmm_launch(P, 0, false) != cudaSuccess)
      rc = set_err(KQ_ERR_BACKEND, "matmul launch");
  }
  if (!rc && cudaMemcpy(y, yd, (size_t)M * a->R * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = set_err(KQ_ERR_BACKEND, "matmul download");
  cudaFree(xd);
  cudaFree(yd);
  cudaFree(xp);
  cudaFree(xs);
  cudaFree(xsum);
  cudaFree(part);
  cudaFree(ticket);
  if (!rc) rc = dev_err_check(a->device);
  return rc;
}

extern "C" int kq_time_matvec(kq_qmat* const* mats, int ncopies, int n, float* ms_out) {
  if (!mats || ncopies < 1 || n < 1 || !ms_out) return set_err(KQ_ERR_ARG, "bad timing arguments");
  kq_qmat* a = mats[0];
  for (int i = 1; i < ncopies; ++i)
    if (!mats[i] || mats[i]->R != a->R || mats[i]->C != a->C || mats[i]->type != a->type || mats[i]->device != a->device)
      return set_err(KQ_ERR_ARG, "timing copies must share shape, type and device");
  CU(cudaSetDevice(a->device));
  float *xd = nullptr, *yd = nullptr;
  CU(cudaMalloc(&xd, (size_t)a->C * 4));
  CU(cudaMalloc(&yd, (size_t)a->R * 4));
  CU(cudaMemset(xd, 0, (size_t)a->C * 4));
  cudaStream_t s;
  CU(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  std::vector<MatvecLaunch> ps(ncopies);
  int rc = KQ_OK;
  for (int i = 0; i < ncopies && !rc; ++i) rc = qmat_gemv_params(mats[i], xd, yd, ps[i]);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  for (int i = 0; i < 3 * ncopies && !rc; ++i)
    if (matvec_launch(ps[i % ncopies], s, false) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "timing launch");
  cudaEventRecord(e0, s);
  for (int i = 0; i < n && !rc; ++i)
    if (matvec_launch(ps[i % ncopies], s, true) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "timing launch");
  cudaEventRecord(e1, s);
  cudaEventSynchronize(e1);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, e0, e1);
  *ms_out = ms / (float)n;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaStreamDestroy(s);
  cudaFree(xd);
  cudaFree(yd);
  if (!rc) rc = dev_err_check(a->device);
  return rc;
}

// ------------------------------------------------------------------------------ the MLP block
// Config-1's block on M rows of a layer's weights (the reference's ffn(), kcpu4.c:287-295, without
// its residual add): xn = rmsnorm(x) * ffn_norm, m = silu(gate xn) * (up xn), y = down m.
// M = 1: the decode graph's two GEMVs (norm in the gate/up prologue, SwiGLU in its epilogue);
// M >= 2: the batched pass (k_bnorm, then the tensor-core GEMM of gate/up with the SwiGLU
// epilogue writing the packed input of the down GEMM). x_dev is read and rewritten unchanged by
// the batched norm; y_dev receives M x dim floats.
static int ffn_block_enqueue(kq_model* m, int layer, float* x_dev, int M, float* y_dev, bool pdl) {
  const kq_config& c = m->c;
  LayerW& w = m->L[layer];
  cudaStream_t s = m->stream;
  if (M == 1) {
    StepOp g1, g2;
    const SegSpec sg[1] = {{w.gu, EPI_SWIGLU, m->mbuf, nullptr}};
    const SegSpec sd[1] = {{w.down, EPI_F32, y_dev, nullptr}};
    int rc = fill_gemv(sg, 1, true, m->nsm, g1.g, g1.pl);
    if (rc || (rc = fill_gemv(sd, 1, false, m->nsm, g2.g, g2.pl))) return rc;
    for (GemvParams* p : {&g1.g, &g2.g}) {
      p->st = m->st; p->vocab = c.vocab; p->hd = c.head_dim; p->ctx = c.ctx; p->err = m->err; p->eps = c.eps;
    }
    g1.g.xmode = XS_NORM; g1.g.h_in = x_dev; g1.g.gamma = w.ffn_norm;
    g2.g.xmode = XS_PLAIN; g2.g.x = m->mbuf;
    CU(launch_gemv(g1.g, g1.pl, s, pdl));
    CU(launch_gemv(g2.g, g2.pl, s, true));
    return KQ_OK;
  }
  BNormParams P;
  std::memset(&P, 0, sizeof(P));
  P.M = M; P.D = c.dim; P.h = x_dev; P.gamma = w.ffn_norm; P.eps = c.eps;
  P.xp = m->bxd; P.xscale = m->bxs_n; P.xsum = m->bxd_sum; P.Npad = (M + 15) & ~15; P.vocab = c.vocab; P.err = m->err;
  CU(launch_pdl(k_bnorm, dim3((unsigned)M), dim3(BN_THREADS), 0, s, P, pdl));
  BatchParams B;
  B.M = M; B.slot = m->bslot; B.rpos = m->brpos; B.mask = m->bmask; B.tree_base = 0; B.seq = nullptr;
  return launch_mlp(m, w, y_dev, B);
}

static int ffn_block_check(kq_model* m, int layer, int M) {
  int rc = model_check(m);
  if (rc || (rc = not_tp(m, "the MLP block"))) return rc;
  if (layer < 0 || layer >= m->c.n_layers) return set_err(KQ_ERR_ARG, "layer out of range");
  if (M < 1 || M > MM_MAXM) return set_err(KQ_ERR_ARG, "rows must be in 1 .. 128");
  if (M > 1 && !batch_supported(m)) return set_err(KQ_ERR_ARG, "the batched pass does not cover this configuration");
  if (M > 1 && (rc = batch_buffers(m))) return rc;
  return KQ_OK;
}

extern "C" int kq_ffn_block(kq_model* m, int layer, const float* x, int M, float* y) {
  int rc = ffn_block_check(m, layer, M);
  if (rc) return rc;
  if (!x || !y) return set_err(KQ_ERR_ARG, "null argument");
  const size_t n = (size_t)M * m->c.dim;
  float *xd = nullptr, *yd = nullptr;
  if (cudaMalloc(&xd, n * 4) != cudaSuccess || cudaMalloc(&yd, n * 4) != cudaSuccess) {
    cudaFree(xd);
    return set_err(KQ_ERR_MEMORY, "MLP block buffers");
  }
  if (cudaMemcpyAsync(xd, x, n * 4, cudaMemcpyHostToDevice, m->stream) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "MLP block upload");
  if (!rc) rc = ffn_block_enqueue(m, layer, xd, M, yd, false);
  if (!rc && cudaMemcpyAsync(y, yd, n * 4, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "MLP block download");
  if (cudaStreamSynchronize(m->stream) != cudaSuccess && !rc) rc = set_err(KQ_ERR_BACKEND, "MLP block");
  cudaFree(xd);
  cudaFree(yd);
  if (!rc) rc = check_dev_err(m);
  return rc;
}

extern "C" int kq_time_ffn_block(kq_model* m, int M, int n, float* ms_out) {
  int rc = ffn_block_check(m, 0, M);
  if (rc) return rc;
  if (n < 1 || !ms_out) return set_err(KQ_ERR_ARG, "bad timing arguments");
  const size_t nx = (size_t)M * m->c.dim;
  float *xd = nullptr, *yd = nullptr;
  if (cudaMalloc(&xd, nx * 4) != cudaSuccess || cudaMalloc(&yd, nx * 4) != cudaSuccess) {
    cudaFree(xd);
    return set_err(KQ_ERR_MEMORY, "MLP block buffers");
  }
  gen_normal_dev(xd, (long long)nx, 0.f, 1.f, 1, 77, m->stream);
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  // successive blocks use successive layers' weights, so a run longer than the layer count
  // streams the whole model's MLP weights (3.1 GB for config-2) instead of an L2-resident layer
  const int L = m->c.n_layers;
  for (int i = 0; i < std::min(n, 2 * L) && !rc; ++i) rc = ffn_block_enqueue(m, i % L, xd, M, yd, i > 0);
  if (!rc && cudaEventRecord(e0, m->stream) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "event");
  for (int i = 0; i < n && !rc; ++i) rc = ffn_block_enqueue(m, i % L, xd, M, yd, true);
  if (!rc && cudaEventRecord(e1, m->stream) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "event");
  if (!rc && cudaEventSynchronize(e1) != cudaSuccess) rc = set_err(KQ_ERR_BACKEND, "MLP block timing");
  float ms = 0.f;
  if (!rc) cudaEventElapsedTime(&ms, e0, e1);
  *ms_out = ms / (float)n;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(xd);
  cudaFree(yd);
  if (!rc) rc = check_dev_err(m);
  return rc;
}

// ------------------------------------------------------------------------------ no-allocation argmax
// kq_qmat_argmax_noalloc runs the argmax form of the GEMV (k_gemv with the ARGMAX epilogue, the
// kernel that closes every decode step) for callers that may not allocate device memory while
// they run. The kernel's scratch -- the row products, one (value, index) partial per CTA, the
// CTAs' completion ticket and the step state the epilogue advances -- is the file-scope array
// below: one fixed-size instance per device, created when the module is loaded, never freed.
// KQ_NOALLOC_MAX_ROWS (include/kq.h, 262144): row products the scratch holds (1 MiB of floats)
constexpr int KQ_NOALLOC_MAX_CTAS = 1024;     // CTA partials the scratch holds
constexpr size_t KQ_NOALLOC_HEADER = 256;     // ticket at 0, DecodeState at 16; zeroed before each launch
constexpr size_t KQ_NOALLOC_VAL = KQ_NOALLOC_HEADER;
constexpr size_t KQ_NOALLOC_IDX = KQ_NOALLOC_VAL + (size_t)KQ_NOALLOC_MAX_CTAS * 4;
constexpr size_t KQ_NOALLOC_PROD = KQ_NOALLOC_IDX + (size_t)KQ_NOALLOC_MAX_CTAS * 4;
constexpr size_t KQ_NOALLOC_BYTES = KQ_NOALLOC_PROD + (size_t)KQ_NOALLOC_MAX_ROWS * 4;
static_assert(16 + sizeof(DecodeState) <= KQ_NOALLOC_HEADER, "scratch header too small");
static_assert(KQ_NOALLOC_PROD % 256 == 0, "row products must stay 256-byte aligned");

static __device__ __align__(256) unsigned char g_noalloc_scratch[KQ_NOALLOC_BYTES];

static unsigned char* g_noalloc_addr[16];   // per device, looked up once
static std::mutex g_noalloc_mu;

// With `device` current: the device address of this device's instance of the scratch array.
static int noalloc_scratch(int device, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_err(KQ_ERR_BACKEND, std::string("kq_qmat_argmax_noalloc: cudaGetSymbolAddress of the scratch: ") +
                                         cudaGetErrorString(e));
    g_noalloc_addr[device] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_addr[device];
  return KQ_OK;
}

extern "C" int kq_qmat_argmax_noalloc(kq_qmat* a, const float* x_dev, int32_t* idx_dev, void* stream) {
  if (!a || !x_dev || !idx_dev) return set_err(KQ_ERR_ARG, "kq_qmat_argmax_noalloc: null argument");
  if (a->R > KQ_NOALLOC_MAX_ROWS)
    return set_err(KQ_ERR_ARG, "kq_qmat_argmax_noalloc: " + std::to_string(a->R) + " rows exceed the static scratch (at most " +
                                   std::to_string(KQ_NOALLOC_MAX_ROWS) + " rows)");
  CU(cudaSetDevice(a->device));
  unsigned char* s = nullptr;
  int rc = noalloc_scratch(a->device, &s);
  if (rc) return rc;
  SegSpec ss[1] = {{a, EPI_ARGMAX, reinterpret_cast<float*>(s + KQ_NOALLOC_PROD), nullptr}};
  GemvParams p;
  GemvPlan pl;
  rc = fill_gemv(ss, 1, false, g_dev[a->device].nsm, p, pl);
  if (rc) return rc;
  if (pl.grid > KQ_NOALLOC_MAX_CTAS)
    return set_err(KQ_ERR_ARG, "kq_qmat_argmax_noalloc: launch needs " + std::to_string(pl.grid) +
                                   " CTA partials, the static scratch holds " + std::to_string(KQ_NOALLOC_MAX_CTAS));
  p.xmode = XS_PLAIN;
  p.x = x_dev;
  p.err = g_dev[a->device].err;
  p.ticket = reinterpret_cast<int*>(s);
  p.st = reinterpret_cast<DecodeState*>(s + 16);
  p.part_val = reinterpret_cast<float*>(s + KQ_NOALLOC_VAL);
  p.part_idx = reinterpret_cast<int*>(s + KQ_NOALLOC_IDX);
  p.out_ids = idx_dev;   // written at st->steps == 0
  p.out_cap = 1;
  // the ticket and the step state must start at zero (a call that failed part-way can leave them set)
  CU(cudaMemsetAsync(s, 0, KQ_NOALLOC_HEADER, (cudaStream_t)stream));
  CU(launch_gemv(p, pl, (cudaStream_t)stream, false));
  return KQ_OK;
}

// ------------------------------------------------------------------------------ prompt-lookup drafter
struct kq_ngram {
  kq::NgramIndex ix;
  kq_ngram(int nmax, int nmin) : ix(nmax, nmin) {}
};
extern "C" kq_ngram* kq_ngram_create(int nmax, int nmin) {
  if (nmin < 1 || nmax < nmin || nmax > 64) {
    set_err(KQ_ERR_ARG, "n-gram sizes must satisfy 1 <= nmin <= nmax <= 64");
    return nullptr;
  }
  try {
    return new kq_ngram(nmax, nmin);
  } catch (...) {
    set_err(KQ_ERR_MEMORY, "n-gram drafter");
    return nullptr;
  }
}
extern "C" void kq_ngram_free(kq_ngram* d) { delete d; }
extern "C" int kq_ngram_reset(kq_ngram* d, const int32_t* hist, int n) {
  if (!d || n < 0 || (n > 0 && !hist)) return set_err(KQ_ERR_ARG, "bad n-gram history");
  try {
    d->ix.reset(hist, n);
  } catch (...) {
    return set_err(KQ_ERR_MEMORY, "n-gram drafter");
  }
  return KQ_OK;
}
extern "C" int kq_ngram_push(kq_ngram* d, int32_t tok) {
  if (!d) return set_err(KQ_ERR_ARG, "null n-gram drafter");
  try {
    d->ix.push(tok);
  } catch (...) {
    return set_err(KQ_ERR_MEMORY, "n-gram drafter");
  }
  return KQ_OK;
}
extern "C" int kq_ngram_truncate(kq_ngram* d, int L) {
  if (!d || L < 0) return set_err(KQ_ERR_ARG, "bad n-gram truncation");
  d->ix.truncate(L);
  return KQ_OK;
}
extern "C" int kq_ngram_propose(kq_ngram* d, int k, int32_t* out) {
  if (!d || k < 0 || (k > 0 && !out)) return set_err(KQ_ERR_ARG, "bad n-gram proposal arguments");
  return d->ix.propose(k, out);
}
extern "C" int kq_ngram_length(const kq_ngram* d) { return d ? d->ix.length() : 0; }
