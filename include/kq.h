/* kq.h -- C ABI of the B200 (sm_100a) Kindi-Q4 decode / speculative-verify runtime.
 *
 * Plain C types only: opaque handles, int status codes (0 = ok, < 0 = error, message from
 * kq_error()), caller-owned host buffers. This mirrors the conventions of the reference's native
 * CPU library (scripts/kindi_q4/kindi/kcpu4.c:303-344: int status returns, caller-owned buffers,
 * an opaque model, sentinel -2 for a backend failure) and the error-string getter of its Metal
 * bridge (scripts/kindi_q4/kindi/metal4.mm:13).
 *
 * Tensor bytes are GGUF block order: row-major [rows][cols/256][block], Q4_K blocks of 144 B and
 * Q6_K blocks of 210 B (type codes 12 and 14, as in the GGUF file and the Kindi pack index).
 */
#ifndef KQ_H
#define KQ_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KQ_Q4_K 12
#define KQ_Q6_K 14

/* Status codes. */
#define KQ_OK            0
#define KQ_ERR_ARG      -1   /* bad argument (reference: ValueError from cpu4.Engine.feed/step) */
#define KQ_ERR_BACKEND  -2   /* CUDA failure (reference: kc_step returns -2, kcpu4.c:334) */
#define KQ_ERR_OVERFLOW -3   /* position past the context (reference: OverflowError, cpu4.py:214-215) */
#define KQ_ERR_MEMORY   -4   /* device allocation failed (reference: MemoryError admission guards) */
#define KQ_ERR_TIMEOUT  -5   /* a bounded device wait gave up; the device flagged an error */

/* Dense GQA decoder configuration (BASELINE config-2 by default, see kq_config_default). */
typedef struct {
  int dim;            /* hidden width D (multiple of 256) */
  int n_layers;
  int n_heads;        /* query heads */
  int n_kv_heads;
  int head_dim;       /* 128 */
  int ffn;            /* SwiGLU width (multiple of 256) */
  int vocab;          /* multiple of 8 */
  int ctx;            /* positions in the K/V cache */
  float rope_theta;
  float eps;          /* RMS norm epsilon */
  int t_q, t_k, t_v, t_o, t_gate, t_up, t_down, t_emb, t_out;   /* KQ_Q4_K / KQ_Q6_K per tensor */
  int max_tokens;     /* widest verify / prefill pass (rows per pass) */
} kq_config;

/* Tensor kinds for kq_model_set_tensor (layer = -1 for the global tensors). */
enum {
  KQ_T_EMB = 0, KQ_T_OUT = 1, KQ_T_OUTNORM = 2,
  KQ_T_ATTN_NORM = 3, KQ_T_Q = 4, KQ_T_K = 5, KQ_T_V = 6, KQ_T_O = 7,
  KQ_T_FFN_NORM = 8, KQ_T_GATE = 9, KQ_T_UP = 10, KQ_T_DOWN = 11
};

typedef struct kq_model kq_model;   /* opaque */
typedef struct kq_qmat kq_qmat;     /* opaque quantised matrix resident on the device */

/* ------------------------------------------------------------------ library */
int kq_version(void);
const char* kq_error(void);                          /* last error of this thread ("" if none) */
int kq_device_count(void);
void kq_config_default(kq_config* cfg);              /* BASELINE config-2 */

/* ------------------------------------------------------------------ model lifecycle
 * Replaces gpu4.Engine.__init__ (scripts/kindi_q4/kindi/gpu4.py:51-90) and make_engine
 * (scripts/kindi_q4/kindi/engine.py:369-381) for the Q4 pack path. */
kq_model* kq_model_create(const kq_config* cfg, int device);   /* NULL on failure, see kq_error */
void kq_model_free(kq_model* m);

/* Kindi Q4 packs (a repacked GGUF directory: kindi_pack.json, index.json, weights.bin in the 8-row
 * interleave, f32.bin; scripts/kindi_q4/kindi/q4pack.py:110-180). The manifest, file sizes,
 * SHA-256 digests (skipped when KINDI_Q4_VERIFY=size), tensor set, shapes, types and spans are
 * checked before anything is allocated, as verify_pack does (q4pack.py:86-108). The manifest's
 * `dimensions` describe the dense GQA decoder (layers, width, ffn, heads, kv_heads, head_dim,
 * rope_dim = head_dim, rope_base, optional norm_eps, full_attention_interval 1); the reference's
 * hybrid GDN profile is rejected with KQ_ERR_ARG.
 * kq_pack_read_config: validate only (no GPU) and return the model configuration for context ctx.
 * kq_model_load_pack: validate, create the model on `device` and upload every tensor (make_engine,
 * engine.py:369-381, with gpu4.Engine's weight upload, gpu4.py:51-90). NULL on failure. */
int kq_pack_read_config(const char* dir, int ctx, kq_config* out);
kq_model* kq_model_load_pack(const char* dir, int ctx, int device);

/* ------------------------------------------------------------------ tensor parallelism
 * One process per GPU. A shard holds KV heads [r*nkv/W, (r+1)*nkv/W) with their query heads
 * (q/k/v rows, o input columns, K/V cache), the FFN slice r (gate/up rows, down input columns) and
 * the vocabulary slice r of the output head; embedding and norms are whole on every rank. The
 * batched pass (kq_feed_batch, kq_verify, kq_step) sums the o and down partials with one NCCL
 * all-reduce each per layer and all-gathers the head's per-rank argmax. Generated shards are
 * bit-identical slices of the whole model kq_model_fill_synthetic generates. Needs n_kv_heads and
 * vocab divisible by W and 256-column slices of ffn and n_heads*head_dim. Not available on a
 * shard: kq_logits, kq_hidden, kq_decode_loop, kq_time_decode, kq_accept, kq_model_set_tensor. */
int kq_tp_unique_id(uint8_t* out128);                 /* ncclGetUniqueId, 128 bytes */
kq_model* kq_model_create_tp(const kq_config* cfg, int device, int rank, int world, const uint8_t* id128);
int kq_model_tp(const kq_model* m, int* rank, int* world);
/* Fill every tensor from the seeded synthetic generator, on the device. */
int kq_model_fill_synthetic(kq_model* m, uint64_t seed);
/* Upload one tensor: quantised tensors as GGUF block bytes, norms as float32 [dim]. */
int kq_model_set_tensor(kq_model* m, int layer, int kind, const void* host, size_t bytes);
/* Engine.reset (cpu4.py:207-209): clears the K/V cache. */
int kq_model_reset(kq_model* m);
/* Fill the K/V cache of every layer at positions [0, npos) with seeded fp16 ~ N(0,1). */
int kq_model_fill_kv(kq_model* m, int npos, uint64_t seed);
/* Copy one layer's K (which = 0) or V (which = 1) cache rows [0, npos) to the host in the
 * reference order [pos][kv][head_dim] (kcpu4.c:239-241). */
int kq_model_get_kv(kq_model* m, int layer, int which, int npos, uint16_t* out);

/* ------------------------------------------------------------------ engine API
 * Engine.feed / Engine.step / Engine.generate (cpu4.py:211-236; engine.py:308-366), the
 * equivalents of kc_step(model, tok, pos, head) (kcpu4.c:303). */
int kq_feed(kq_model* m, int tok, int pos);          /* 0, or an error code */
int kq_step(kq_model* m, int tok, int pos);          /* greedy next token id, or an error code */
int kq_feed_batch(kq_model* m, const int32_t* toks, int n, int pos);
int kq_generate(kq_model* m, const int32_t* ids, int n_ids, int n, int32_t* out);
/* Engine.ylog (engine.py:323-331): the logits of the last step (row 0) or verify row `row`. */
int kq_logits(kq_model* m, int row, float* out);
/* Hidden residual stream after the last step (kcpu4.c:331: h), dim floats. */
int kq_hidden(kq_model* m, float* out);

/* Device-resident greedy decode: n steps, each feeding the previous step's argmax, starting
 * from (tok, pos); no host round trip between steps. Writes the n ids to out. */
int kq_decode_loop(kq_model* m, int tok, int pos, int n, int32_t* out);
/* Time n device-resident decode steps (CUDA events on the model's stream); returns ms. */
int kq_time_decode(kq_model* m, int tok, int pos, int n, float* ms_out);
/* Kernels one decode step launches (the kernel nodes of the step's CUDA graph; 1 for the
 * persistent form), or < 0 on error. A measurement hook with no reference counterpart: the
 * reference's CuPy engine launches its kernels one by one from Python (gpu4.py:50-110). */
int kq_step_kernels(kq_model* m);
/* Time split of the batched passes (prefill, verify, batched decode) since the last call, in ms:
 * [0] tensor-core GEMMs and their activation packing, [1] attention, [2] NCCL all-reduces,
 * [3] norms, head argmax and the rest; then resets. Only for a model created with
 * KQ_PHASE_TIMES=1 in the environment (an event separates every launch group, so the passes run
 * without programmatic launch overlap). A measurement hook with no reference counterpart. */
int kq_phase_times(kq_model* m, float* ms4);

/* ------------------------------------------------------------------ speculative verification
 * Draft-then-verify over a draft TREE (the reference verifies linear chains only: spec.py:790-793
 * greedy chain, spec.py:769-787 acceptance, spec.py:531-542 commit). A tree of n <= KQ_MAX_TREE
 * nodes is given by parent pointers: node 0 is the last accepted token (at position pos, not yet
 * fed), parents[0] = -1 and 0 <= parents[i] < i; a linear chain is parents[i] = i - 1. */
#define KQ_MAX_TREE 128
/* Runs every node through the model. Node i's K/V go to cache slot pos + i, its rotary position is
 * pos + depth(i), and it attends to the positions below pos and to its ancestors and itself.
 * Optional outputs: logits (n x vocab floats) and best (n argmax ids, lowest id on ties).
 * The logits stay on the device for kq_accept. */
int kq_verify(kq_model* m, const int32_t* tokens, const int32_t* parents, int n, int pos, float* logits,
              int32_t* best);
/* Accepts a prefix path of the tree verified by the last kq_verify (same tokens / parents), on the
 * device. temperature 0: greedy (a child is accepted iff its token is the argmax of its parent's
 * logits; the last node's argmax is emitted). temperature > 0: speculative sampling with target
 * softmax(logits / T) and draft distributions softmax(draft_logits[v]) (n x vocab, row v: the
 * distribution v's children were drawn from): child c accepted iff u_acc[c] * q(d_c) < p(d_c),
 * recursive residuals max(0, p - q) on rejection, final token by inverse CDF at u_fin[v]
 * (uniforms in [0,1), one per node). Writes the accepted node path (path[0] = 0; *path_len
 * entries) and the emitted tokens (accepted drafts, then one sampled token). Returns the number
 * of emitted tokens. The CPU oracle's or_accept computes the identical result. */
int kq_accept(kq_model* m, const int32_t* tokens, const int32_t* parents, int n, const float* draft_logits,
              float temperature, const float* u_acc, const float* u_fin, int32_t* path, int32_t* out,
              int32_t* path_len);
/* Draft distributions resident on the device (a drafter on the GPU writes its logits there):
 * kq_draft_logits gives the model's buffer (KQ_MAX_TREE rows of `ld` = vocab floats, row v = the
 * distribution v's children were drawn from), kq_draft_upload fills rows [0, n) from the host,
 * and kq_accept_resident is kq_accept reading the draft logits from that buffer. */
int kq_draft_logits(kq_model* m, float** dev, int* ld);
int kq_draft_upload(kq_model* m, const float* host, int n);
int kq_accept_resident(kq_model* m, const int32_t* tokens, const int32_t* parents, int n, float temperature,
                       const float* u_acc, const float* u_fin, int32_t* path, int32_t* out, int32_t* path_len);
/* K/V compaction: the K/V rows of path[1..k] (increasing node ids, path[0] = 0) move from slots
 * pos + path[j] to positions pos + j, so the accepted tokens sit at consecutive positions. */
int kq_commit(kq_model* m, const int32_t* path, int k, int pos);

/* ------------------------------------------------------------------ batched decode of many sequences
 * Config-4 decode (no counterpart in the reference's Q4 path, which decodes one sequence): every
 * sequence has its own K/V cache ([n_kv][ctx][hd] per layer and tensor, on a tensor-parallel
 * shard its own KV heads), and a step takes one token per sequence through the batched pass, so
 * the weights stream once for all of them. kq_batch_caches allocates the caches (zeroed) for
 * n_seq sequences; kq_batch_feed prefills sequence `seq` from `pos`; kq_batch_step runs one token
 * of each of n <= 128 distinct sequences (token toks[i] at position pos[i] of sequence seqs[i],
 * attending to [0, pos[i]]) and writes their greedy ids to out. */
int kq_batch_caches(kq_model* m, int n_seq);
int kq_batch_feed(kq_model* m, int seq, const int32_t* toks, int n, int pos);
int kq_batch_step(kq_model* m, const int32_t* seqs, const int32_t* toks, const int32_t* pos, int n, int32_t* out);

/* ------------------------------------------------------------------ matrix hooks
 * kc_matvec / kc_dequant equivalents (kcpu4.c:337-341, q4kernels.h:12-36). */
kq_qmat* kq_qmat_create(int type, int rows, int cols, int device);
void kq_qmat_free(kq_qmat* a);
int kq_qmat_upload(kq_qmat* a, const void* gguf_bytes, size_t bytes);
int kq_qmat_fill_synthetic(kq_qmat* a, uint64_t seed, uint64_t stream);
/* Bit-exact dequantisation of `nrows` rows starting at `row` into host floats (q4_decode). */
int kq_qmat_dequant(kq_qmat* a, int row, int nrows, float* out);
/* y[r] = sum_c W[r][c] x[c] for host x (cols floats) and host y (rows floats). */
int kq_qmat_matvec(kq_qmat* a, const float* x, float* y);
/* M-token product Y[m][r] = sum_c W[r][c] X[m][c] (host buffers, M <= 64). */
int kq_qmat_matmul(kq_qmat* a, const float* x, int M, float* y);
/* Device-pointer variants on a CUDA stream (0 = legacy default), no synchronisation. */
int kq_qmat_matvec_dev(kq_qmat* a, const float* x_dev, float* y_dev, void* stream);
/* Time n launches of the matvec on device buffers, rotating over `ncopies` matrices (so the
 * weights are re-read from HBM); returns the mean launch ms measured with CUDA events. */
int kq_time_matvec(kq_qmat* const* mats, int ncopies, int n, float* ms_out);

/* ------------------------------------------------------------------ the MLP block (config-1)
 * The feed-forward block of layer `layer` on M rows (1 <= M <= 128), the reference's ffn()
 * (kcpu4.c:287-295) without its residual add: xn = rmsnorm(x) * ffn_norm (fp64 sum of squares,
 * kcpu4.c:123-139), m = silu(gate xn) * (up xn) (kcpu4.c:292), y = down m. The reference runs it
 * as M separate token steps (kc_matvec per matrix); here M = 1 is the decode GEMV pair and M >= 2
 * one batched tensor-core pass. x and y are host [M][dim] floats. Whole models only. */
int kq_ffn_block(kq_model* m, int layer, const float* x, int M, float* y);
/* Time n blocks of M rows on device buffers, block i on layer i % n_layers (the weights stream
 * from HBM); mean ms per block from CUDA events. */
int kq_time_ffn_block(kq_model* m, int M, int n, float* ms_out);
/* Bytes the device layout of this matrix occupies (equal to the GGUF bytes). */
size_t kq_qmat_bytes(const kq_qmat* a);

/* ------------------------------------------------------------------ no-allocation argmax
 * This entry point has no counterpart in the reference; it is an addition of this library.
 *
 * *idx_dev = the lowest row index r with the largest (W x)[r], for device x_dev (cols floats);
 * the same GEMV and tie rule as the greedy head of kq_step, enqueued on `stream` (0 = legacy
 * default) without synchronising. It is for callers that may not allocate device memory while
 * they run: a server that hands all free HBM to its K/V cache at start-up (an allocation would
 * fail or evict), or a latency-bound sampling loop that cannot take the device-wide
 * synchronisation cudaMalloc / cudaFree may imply. The call allocates nothing: the kernel's
 * scratch (the row products, the per-CTA partials and a completion ticket) is a fixed array
 * inside this library, one per device, KQ_NOALLOC_MAX_ROWS row products at most.
 *  - Matrices with more than KQ_NOALLOC_MAX_ROWS rows are rejected with KQ_ERR_ARG.
 *  - The first call on each device looks up that device's scratch address (cudaGetSymbolAddress);
 *    make it before any stream capture that could include this call.
 *  - There is one scratch per device: calls on the same device that overlap in time (different
 *    streams, or different host threads) race and give wrong indices. Calls one after another on
 *    one stream are safe.
 *  - A bounded-wait failure on the device is reported, as for kq_qmat_matvec_dev, by the next
 *    synchronising matrix call (KQ_ERR_TIMEOUT). */
#define KQ_NOALLOC_MAX_ROWS 262144
int kq_qmat_argmax_noalloc(kq_qmat* a, const float* x_dev, int32_t* idx_dev, void* stream);

/* ------------------------------------------------------------------ prompt-lookup drafter
 * Replaces NgramDraft (scripts/kindi_q4/kindi/spec.py:801-841): the tokens that followed the
 * latest earlier occurrence of the longest matching suffix of the history, suffix lengths
 * nmax .. nmin; -1 marks an unknown token (a suffix holding one is skipped, a continuation holding
 * one gives no proposal). Host-side only (no GPU). A proposal of k tokens is a draft chain for
 * kq_verify: tokens [last, d0, .., d(k-1)], parents [-1, 0, .., k-1].
 *  kq_ngram_create    nmax >= nmin >= 1, nmax <= 64 (NgramDraft(nmax=4, nmin=1) by default there);
 *                     null (kq_error) on bad sizes
 *  kq_ngram_reset     NgramDraft.reset(hist): the history is replaced by hist[0..n)
 *  kq_ngram_push      NgramDraft.push(t)
 *  kq_ngram_truncate  NgramDraft.truncate(L): drop positions >= L (L >= 0)
 *  kq_ngram_propose   NgramDraft.propose(k): writes up to k tokens to out and returns how many
 *                     (k >= 0), or a negative KQ_ERR_* code
 *  kq_ngram_length    tokens in the history */
typedef struct kq_ngram kq_ngram;
kq_ngram* kq_ngram_create(int nmax, int nmin);
void kq_ngram_free(kq_ngram* d);
int kq_ngram_reset(kq_ngram* d, const int32_t* hist, int n);
int kq_ngram_push(kq_ngram* d, int32_t tok);
int kq_ngram_truncate(kq_ngram* d, int L);
int kq_ngram_propose(kq_ngram* d, int k, int32_t* out);
int kq_ngram_length(const kq_ngram* d);

#ifdef __cplusplus
}
#endif
#endif
