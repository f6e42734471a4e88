/* kq_oracle.c -- CPU ORACLE FOR TESTS ONLY.
 *
 * This file is test infrastructure: a plain-C restatement of the Kindi Q4 CPU path that the
 * CUDA library is checked against. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm load it. The product library (libkq.so) never links or calls it.
 *
 * What it restates (paths relative to the reference project root):
 *   - Q4_K / Q6_K block decode ............ scripts/kindi_q4/kindi/q4kernels.h:12-33
 *   - row decode .......................... scripts/kindi_q4/kindi/q4kernels.h:34-36
 *   - fused dequant dot, AVX2 lane order ... scripts/kindi_q4/kindi/q4kernels.h:37-71
 *   - tiled block addressing .............. scripts/kindi_q4/kindi/q4kernels.h:8-10
 *   - matvec over rows .................... scripts/kindi_q4/kindi/kcpu4.c:337-340
 *   - residual add + fp64 RMS norm ........ scripts/kindi_q4/kindi/kcpu4.c:123-139
 *   - RoPE tables (fp64 -> f32) ........... scripts/kindi_q4/kindi/cpu4.py:175-178
 *   - NeoX rotary ......................... scripts/kindi_q4/kindi/kcpu4.c:223-236
 *   - fp16 K/V store, scores, softmax, P.V  scripts/kindi_q4/kindi/kcpu4.c:239-282
 *   - SwiGLU FFN .......................... scripts/kindi_q4/kindi/kcpu4.c:287-295
 *   - output head + strict-> argmax ....... scripts/kindi_q4/kindi/kcpu4.c:316-327
 * The dense GQA decoder (32 q / 8 kv heads of 128, no q/k norm, no output gate, full-width
 * RoPE) is the BASELINE config-2 model, which the reference's kc_step cannot run (it is wired
 * to the hybrid GDN model); it is assembled here from the reference's building blocks above.
 *
 * Parity pins: or_decode_block and or_matvec are checked bit-for-bit against the reference's
 * own kc_dequant / kc_matvec (compiled from the reference sources into oracle/_ref) and against
 * the golden vectors in tests/golden, which were produced by the reference's numpy decoder
 * (q4pack.py:52-76) and kc_matvec. or_ffn_block is checked bit-for-bit against the reference's
 * ffn, and the embedding row, final norm, head and argmax of a step against the reference's
 * kc_step on a model of no layers (oracle/ref_blocks.c over the unmodified kcpu4.c). or_accept
 * is checked in distribution against the reference's spec_accept (spec.py:769-787). The dense
 * attention and the layer composition are pinned to this restatement only (parity unpinned
 * there: the reference's attention is the hybrid model's gated form).
 *
 * Build flags follow cpu4.py:65-66 (-O3 -ffp-contract=off -fno-math-errno -fopenmp).
 */
#include <stdint.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_Q4K 12
#define OR_Q6K 14

/* ------------------------------------------------------------------ fp16 (IEEE binary16, RNE) */
/* Equivalent of the reference's _cvtsh_ss / _cvtss_sh(f, 0) (kcpu4.c:60-73), written with
 * the compiler's _Float16 type so it needs no F16C. */
float or_h2f(uint16_t h){ _Float16 v; memcpy(&v, &h, 2); return (float)v; }
uint16_t or_f2h(float f){ _Float16 v = (_Float16)f; uint16_t h; memcpy(&h, &v, 2); return h; }

/* ------------------------------------------------------------------ matrices */
typedef struct {
  const uint8_t* W;   /* quantised blocks */
  int R, C, type;     /* rows, columns (multiple of 256), 12 = Q4_K, 14 = Q6_K */
  int layout;         /* 0: GGUF row-major [R][C/256][block]; 1: Kindi pack [R/8][C/256][8][block] */
} OMat;

int or_block_bytes(int type){ return type == OR_Q4K ? 144 : 210; }

/* q4kernels.h:8-10 for layout 1; plain row-major addressing for layout 0. */
const uint8_t* or_block(const OMat* a, int row, int g){
  const size_t G = (size_t)(a->C / 256), bs = (size_t)or_block_bytes(a->type);
  if(a->layout == 1) return a->W + ((((size_t)(row / 8)) * G + (size_t)g) * 8 + (size_t)(row % 8)) * bs;
  return a->W + ((size_t)row * G + (size_t)g) * bs;
}

static uint16_t or_u16(const uint8_t* p){ uint16_t v; memcpy(&v, p, 2); return v; }

/* q4kernels.h:12-33. Exact products in the reference's order: w = fl(fl(d*sc)*q) - fl(dmin*mn)
 * for Q4_K and w = fl(d*scale)*(q-32) for Q6_K. */
void or_decode_block(const uint8_t* b, int type, float* y){
  if(type == OR_Q4K){
    const float d = or_h2f(or_u16(b)), dm = or_h2f(or_u16(b + 2));
    const uint8_t* s = b + 4;
    for(int k = 0; k < 8; k++){
      const int sc = k < 4 ? (s[k] & 63) : ((s[k + 4] & 15) | ((s[k - 4] >> 6) << 4));
      const int mn = k < 4 ? (s[k + 4] & 63) : ((s[k + 4] >> 4) | ((s[k] >> 6) << 4));
      const float ds = d * (float)sc, ms = dm * (float)mn;
      const uint8_t* q = b + 16 + (k / 2) * 32;
      for(int j = 0; j < 32; j++){
        const float qf = (float)((q[j] >> ((k % 2) * 4)) & 15);
        const float t = ds * qf;
        y[k * 32 + j] = t - ms;
      }
    }
  } else {
    const float d = or_h2f(or_u16(b + 208));
    const int8_t* s = (const int8_t*)(b + 192);
    for(int h = 0; h < 2; h++) for(int k = 0; k < 4; k++) for(int j = 0; j < 32; j++){
      const int low = (b[h * 64 + (k % 2) * 32 + j] >> ((k / 2) * 4)) & 15;
      const int high = (b[128 + h * 32 + j] >> (2 * k)) & 3;
      const float ds = d * (float)s[h * 8 + k * 2 + j / 16];
      y[h * 128 + k * 32 + j] = ds * (float)((low | (high << 4)) - 32);
    }
  }
}

/* q4kernels.h:34-36 */
void or_dequant_row(const OMat* a, int row, float* y){
  for(int g = 0; g < a->C / 256; g++) or_decode_block(or_block(a, row, g), a->type, y + g * 256);
}

/* q4kernels.h:37-71, the AVX2 branch, restated lane by lane: eight fp32 accumulators, lane l
 * takes element (8*i + l) of each 8-wide step in (block, sub-block, j) order; products and sums
 * are separately rounded (the reference builds with -ffp-contract=off); the lanes are added
 * 0..7 at the end. The result is bit-identical to the reference's kc_matvec on x86 with AVX2. */
float or_dot(const OMat* a, int row, const float* x){
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int G = a->C / 256;
  for(int g = 0; g < G; g++){
    const uint8_t* b = or_block(a, row, g);
    const float* in = x + 256 * g;
    if(a->type == OR_Q4K){
      const float d = or_h2f(or_u16(b)), dm = or_h2f(or_u16(b + 2));
      const uint8_t* s = b + 4;
      for(int k = 0; k < 8; k++){
        const int sc = k < 4 ? (s[k] & 63) : ((s[k + 4] & 15) | ((s[k - 4] >> 6) << 4));
        const int mn = k < 4 ? (s[k + 4] & 63) : ((s[k + 4] >> 4) | ((s[k] >> 6) << 4));
        const float ds = d * (float)sc, ms = dm * (float)mn;
        const uint8_t* q = b + 16 + (k / 2) * 32;
        for(int j = 0; j < 32; j += 8)
          for(int l = 0; l < 8; l++){
            const float qf = (float)((q[j + l] >> ((k & 1) * 4)) & 15);
            const float t = ds * qf;
            const float w = t - ms;
            const float p = w * in[k * 32 + j + l];
            acc[l] = acc[l] + p;
          }
      }
    } else {
      const float d = or_h2f(or_u16(b + 208));
      const int8_t* s = (const int8_t*)(b + 192);
      for(int h = 0; h < 2; h++) for(int k = 0; k < 4; k++) for(int j = 0; j < 32; j += 8){
        const float ds = d * (float)s[h * 8 + k * 2 + j / 16];
        for(int l = 0; l < 8; l++){
          const int low = (b[h * 64 + (k % 2) * 32 + j + l] >> ((k / 2) * 4)) & 15;
          const int high = (b[128 + h * 32 + j + l] >> (2 * k)) & 3;
          const float w = ds * (float)((low | (high << 4)) - 32);
          const float p = w * in[h * 128 + k * 32 + j + l];
          acc[l] = acc[l] + p;
        }
      }
    }
  }
  float total = 0.f;
  for(int l = 0; l < 8; l++) total += acc[l];
  return total;
}

/* kcpu4.c:337-340: rows split across threads; each row is one sequential or_dot, so the result
 * does not depend on the thread count. */
void or_matvec(const OMat* a, const float* x, float* y){
  #pragma omp parallel for schedule(static)
  for(int r = 0; r < a->R; r++) y[r] = or_dot(a, r, x);
}

/* Convenience for ctypes callers: matvec with the matrix given by its fields. */
void or_matvec_raw(const uint8_t* W, int R, int C, int type, int layout, const float* x, float* y){
  OMat a = {W, R, C, type, layout};
  or_matvec(&a, x, y);
}
void or_dequant_raw(const uint8_t* W, int R, int C, int type, int layout, int row, float* y){
  OMat a = {W, R, C, type, layout};
  or_dequant_row(&a, row, y);
}

/* ------------------------------------------------------------------ seeded synthetic data
 * Counter-based generator shared (as a specification) with the CUDA library's on-device
 * synthetic fill: draw i of stream s under seed S is splitmix64's output function applied to
 * base(S, s) + (i + 1) * GAMMA. Every value below is derived from those 64-bit draws with exact
 * integer work or IEEE fp32 operations without contraction, so host and device agree bit for bit.
 */
#define OR_GAMMA 0x9E3779B97F4A7C15ull
static inline uint64_t or_fin(uint64_t z){
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
uint64_t or_base(uint64_t seed, uint64_t stream){ return or_fin(or_fin(seed * OR_GAMMA + 0x632BE59BD9B4E019ull) ^ (stream * 0xD1B54A32D192ED03ull)); }
static inline uint64_t or_draw(uint64_t base, uint64_t i){ return or_fin(base + (i + 1) * OR_GAMMA); }

/* U[lo, lo + span) from 24 bits: lo + (u * 2^-24) * span, two roundings. */
static inline float or_unif24(uint32_t u24, float lo, float span){
  const float u = (float)u24 * 0x1p-24f;
  const float t = u * span;
  return lo + t;
}
/* Approximately N(0,1): Irwin-Hall sum of twelve 24-bit uniforms minus 6, formed exactly in
 * integers and rounded once to fp32. */
static inline float or_nrm(uint64_t base, uint64_t i){
  int64_t s = 0;
  for(int k = 0; k < 6; k++){
    const uint64_t r = or_draw(base, i * 6 + (uint64_t)k);
    s += (int64_t)(r & 0xFFFFFF) + (int64_t)((r >> 24) & 0xFFFFFF);
  }
  return (float)(s - 6ll * 16777216ll) * 0x1p-24f;
}

/* Q4_K block number bi of a stream (19 draws): d, dmin ~ U[1e-4, 4e-4] (fp16), eight 6-bit
 * scales and eight 6-bit mins ~ U{0..63} packed as q4kernels.h:17-18 unpacks them, 128 random
 * nibble bytes. */
void or_gen_q4k_block(uint64_t base, uint64_t bi, uint8_t* b){
  const uint64_t k0 = bi * 19;
  const uint64_t r0 = or_draw(base, k0), r1 = or_draw(base, k0 + 1), r2 = or_draw(base, k0 + 2);
  const uint16_t d = or_f2h(or_unif24((uint32_t)(r0 & 0xFFFFFF), 1e-4f, 3e-4f));
  const uint16_t dm = or_f2h(or_unif24((uint32_t)((r0 >> 24) & 0xFFFFFF), 1e-4f, 3e-4f));
  memcpy(b, &d, 2); memcpy(b + 2, &dm, 2);
  int sc[8], mn[8];
  for(int k = 0; k < 8; k++){ sc[k] = (int)((r1 >> (8 * k)) & 63); mn[k] = (int)((r2 >> (8 * k)) & 63); }
  uint8_t* s = b + 4;
  for(int k = 0; k < 4; k++){
    s[k] = (uint8_t)(sc[k] | ((sc[k + 4] >> 4) << 6));
    s[k + 4] = (uint8_t)(mn[k] | ((mn[k + 4] >> 4) << 6));
    s[k + 8] = (uint8_t)((sc[k + 4] & 15) | ((mn[k + 4] & 15) << 4));
  }
  for(int w = 0; w < 16; w++){ const uint64_t r = or_draw(base, k0 + 3 + (uint64_t)w); memcpy(b + 16 + 8 * w, &r, 8); }
}

/* Q6_K block number bi (27 draws): ql[128], qh[64] random bytes, int8 scales ~ U{-64..63},
 * d ~ U[1e-4, 4e-4] (fp16). */
void or_gen_q6k_block(uint64_t base, uint64_t bi, uint8_t* b){
  const uint64_t k0 = bi * 27;
  for(int w = 0; w < 24; w++){ const uint64_t r = or_draw(base, k0 + (uint64_t)w); memcpy(b + 8 * w, &r, 8); }
  const uint64_t s0 = or_draw(base, k0 + 24), s1 = or_draw(base, k0 + 25), rd = or_draw(base, k0 + 26);
  for(int i = 0; i < 16; i++){
    const uint64_t r = i < 8 ? s0 : s1;
    b[192 + i] = (uint8_t)(int8_t)((int)((r >> (8 * (i & 7))) & 127) - 64);
  }
  const uint16_t d = or_f2h(or_unif24((uint32_t)(rd & 0xFFFFFF), 1e-4f, 3e-4f));
  memcpy(b + 208, &d, 2);
}

/* A whole matrix R x C of the given type, in the given layout (0 GGUF row-major, 1 Kindi pack).
 * Block (row, g) is block number row*G + g of the stream whatever the layout. */
void or_gen_matrix(uint8_t* W, int R, int C, int type, int layout, uint64_t seed, uint64_t stream){
  const uint64_t base = or_base(seed, stream);
  const int G = C / 256;
  OMat a = {W, R, C, type, layout};
  #pragma omp parallel for schedule(static)
  for(int row = 0; row < R; row++)
    for(int g = 0; g < G; g++){
      uint8_t* b = (uint8_t*)or_block(&a, row, g);
      const uint64_t bi = (uint64_t)row * (uint64_t)G + (uint64_t)g;
      if(type == OR_Q4K) or_gen_q4k_block(base, bi, b); else or_gen_q6k_block(base, bi, b);
    }
}

/* n values mu + sigma * z, z ~ approx N(0,1) as above (two roundings). */
void or_gen_normal(float* y, int64_t n, float mu, float sigma, uint64_t seed, uint64_t stream){
  const uint64_t base = or_base(seed, stream);
  #pragma omp parallel for schedule(static)
  for(int64_t i = 0; i < n; i++){ const float t = sigma * or_nrm(base, (uint64_t)i); y[i] = mu + t; }
}
/* n token ids ~ U{0..V-1}: ((draw >> 32) * V) >> 32. */
void or_gen_tokens(int32_t* y, int64_t n, int V, uint64_t seed, uint64_t stream){
  const uint64_t base = or_base(seed, stream);
  for(int64_t i = 0; i < n; i++) y[i] = (int32_t)(((or_draw(base, (uint64_t)i) >> 32) * (uint64_t)V) >> 32);
}
/* n uniforms in [0,1) with 24 bits: (draw >> 40) * 2^-24. */
void or_gen_uniform(float* y, int64_t n, uint64_t seed, uint64_t stream){
  const uint64_t base = or_base(seed, stream);
  for(int64_t i = 0; i < n; i++) y[i] = (float)(or_draw(base, (uint64_t)i) >> 40) * 0x1p-24f;
}
/* n random fp16 bit patterns of values ~ N(0,1) (for pre-filled K/V caches). */
void or_gen_half_normal(uint16_t* y, int64_t n, uint64_t seed, uint64_t stream){
  const uint64_t base = or_base(seed, stream);
  #pragma omp parallel for schedule(static)
  for(int64_t i = 0; i < n; i++) y[i] = or_f2h(or_nrm(base, (uint64_t)i));
}

/* ------------------------------------------------------------------ dense GQA decoder (config-2) */
/* Tensor kinds; the synthetic stream of tensor kind k in layer l is (l + 1) * 32 + k, and
 * (0 * 32 + k) for the global tensors. These numbers are part of the shared specification. */
enum { OR_T_EMB = 0, OR_T_OUT = 1, OR_T_OUTNORM = 2,
       OR_T_ATTN_NORM = 3, OR_T_Q = 4, OR_T_K = 5, OR_T_V = 6, OR_T_O = 7,
       OR_T_FFN_NORM = 8, OR_T_GATE = 9, OR_T_UP = 10, OR_T_DOWN = 11 };

typedef struct {
  int D, NL, NH, NKV, HD, NFF, vocab, ctx;
  float rope_theta, eps;
  int t_q, t_k, t_v, t_o, t_gate, t_up, t_down, t_emb, t_out;   /* 12 / 14 per tensor */
} OCfg;

typedef struct {
  OMat q, k, v, o, gate, up, down;
  float *attn_norm, *ffn_norm;
  uint16_t *Kc, *Vc;    /* [ctx][NKV][HD] fp16, kcpu4.c:239-241 */
} OLayer;

typedef struct {
  OCfg c;
  OLayer* L;
  OMat emb, out;
  float* out_norm;
  float *cos_t, *sin_t;           /* [ctx][HD/2] */
  float *h, *y, *xn, *q, *k, *v, *qr, *kr, *sc, *att, *g, *u, *m, *logits;
  int layout;
} OModel;

static uint64_t or_stream(int layer, int kind){ return (uint64_t)(layer + 1) * 32u + (uint64_t)kind; }

static size_t or_mat_bytes(int R, int C, int type){ return (size_t)R * (size_t)(C / 256) * (size_t)or_block_bytes(type); }

static void or_mat_init(OMat* a, int R, int C, int type, int layout, uint64_t seed, uint64_t stream, int gen){
  uint8_t* W = (uint8_t*)malloc(or_mat_bytes(R, C, type));
  a->W = W; a->R = R; a->C = C; a->type = type; a->layout = layout;
  if(gen) or_gen_matrix(W, R, C, type, layout, seed, stream);
}

/* Creates the model with every tensor generated from `seed` (layout 0 or 1 for the quantised
 * blocks). Returns NULL on allocation failure. */
OModel* or_model_create(const OCfg* cfg, uint64_t seed, int layout){
  OModel* m = (OModel*)calloc(1, sizeof(OModel));
  if(!m) return NULL;
  m->c = *cfg; m->layout = layout;
  const OCfg* c = &m->c;
  const int D = c->D, QD = c->NH * c->HD, KD = c->NKV * c->HD, F = c->NFF;
  m->L = (OLayer*)calloc((size_t)c->NL, sizeof(OLayer));
  for(int l = 0; l < c->NL; l++){
    OLayer* L = m->L + l;
    or_mat_init(&L->q, QD, D, c->t_q, layout, seed, or_stream(l, OR_T_Q), 1);
    or_mat_init(&L->k, KD, D, c->t_k, layout, seed, or_stream(l, OR_T_K), 1);
    or_mat_init(&L->v, KD, D, c->t_v, layout, seed, or_stream(l, OR_T_V), 1);
    or_mat_init(&L->o, D, QD, c->t_o, layout, seed, or_stream(l, OR_T_O), 1);
    or_mat_init(&L->gate, F, D, c->t_gate, layout, seed, or_stream(l, OR_T_GATE), 1);
    or_mat_init(&L->up, F, D, c->t_up, layout, seed, or_stream(l, OR_T_UP), 1);
    or_mat_init(&L->down, D, F, c->t_down, layout, seed, or_stream(l, OR_T_DOWN), 1);
    L->attn_norm = (float*)malloc(sizeof(float) * (size_t)D);
    L->ffn_norm = (float*)malloc(sizeof(float) * (size_t)D);
    or_gen_normal(L->attn_norm, D, 1.0f, 0.02f, seed, or_stream(l, OR_T_ATTN_NORM));
    or_gen_normal(L->ffn_norm, D, 1.0f, 0.02f, seed, or_stream(l, OR_T_FFN_NORM));
    L->Kc = (uint16_t*)calloc((size_t)c->ctx * (size_t)KD, 2);
    L->Vc = (uint16_t*)calloc((size_t)c->ctx * (size_t)KD, 2);
  }
  or_mat_init(&m->emb, c->vocab, D, c->t_emb, layout, seed, or_stream(-1, OR_T_EMB), 1);
  or_mat_init(&m->out, c->vocab, D, c->t_out, layout, seed, or_stream(-1, OR_T_OUT), 1);
  m->out_norm = (float*)malloc(sizeof(float) * (size_t)D);
  or_gen_normal(m->out_norm, D, 1.0f, 0.02f, seed, or_stream(-1, OR_T_OUTNORM));
  /* cpu4.py:175-178: inv = theta^(-2i/rope_dim) in fp64, angle table pos*inv in fp64, cast. */
  const int rh = c->HD / 2;
  m->cos_t = (float*)malloc(sizeof(float) * (size_t)c->ctx * (size_t)rh);
  m->sin_t = (float*)malloc(sizeof(float) * (size_t)c->ctx * (size_t)rh);
  for(int p = 0; p < c->ctx; p++)
    for(int i = 0; i < rh; i++){
      const double inv = pow((double)c->rope_theta, -2.0 * (double)i / (double)c->HD);
      const double th = (double)p * inv;
      m->cos_t[(size_t)p * rh + i] = (float)cos(th);
      m->sin_t[(size_t)p * rh + i] = (float)sin(th);
    }
  const int W = D > F ? (D > QD ? D : QD) : (F > QD ? F : QD);
  m->h = (float*)calloc((size_t)D, 4); m->y = (float*)calloc((size_t)D, 4); m->xn = (float*)calloc((size_t)W, 4);
  m->q = (float*)calloc((size_t)QD, 4); m->k = (float*)calloc((size_t)KD, 4); m->v = (float*)calloc((size_t)KD, 4);
  m->qr = (float*)calloc((size_t)QD, 4); m->kr = (float*)calloc((size_t)KD, 4);
  m->sc = (float*)calloc((size_t)c->NH * (size_t)c->ctx, 4); m->att = (float*)calloc((size_t)QD, 4);
  m->g = (float*)calloc((size_t)F, 4); m->u = (float*)calloc((size_t)F, 4); m->m = (float*)calloc((size_t)F, 4);
  m->logits = (float*)calloc((size_t)c->vocab, 4);
  return m;
}

void or_model_free(OModel* m){
  if(!m) return;
  for(int l = 0; l < m->c.NL; l++){
    OLayer* L = m->L + l;
    free((void*)L->q.W); free((void*)L->k.W); free((void*)L->v.W); free((void*)L->o.W);
    free((void*)L->gate.W); free((void*)L->up.W); free((void*)L->down.W);
    free(L->attn_norm); free(L->ffn_norm); free(L->Kc); free(L->Vc);
  }
  free(m->L); free((void*)m->emb.W); free((void*)m->out.W); free(m->out_norm);
  free(m->cos_t); free(m->sin_t);
  free(m->h); free(m->y); free(m->xn); free(m->q); free(m->k); free(m->v); free(m->qr); free(m->kr);
  free(m->sc); free(m->att); free(m->g); free(m->u); free(m->m); free(m->logits);
  free(m);
}

void or_model_reset(OModel* m){
  const size_t kv = (size_t)m->c.ctx * (size_t)m->c.NKV * (size_t)m->c.HD;
  for(int l = 0; l < m->c.NL; l++){ memset(m->L[l].Kc, 0, kv * 2); memset(m->L[l].Vc, 0, kv * 2); }
}

/* Fill the K/V caches of every layer at positions [0, npos) with fp16 ~ N(0,1) values from
 * stream (layer+1)*32+12 (K) and +13 (V) under `seed`, in [pos][kv][hd] order. */
void or_model_fill_kv(OModel* m, int npos, uint64_t seed){
  const int64_t n = (int64_t)npos * m->c.NKV * m->c.HD;
  for(int l = 0; l < m->c.NL; l++){
    or_gen_half_normal(m->L[l].Kc, n, seed, or_stream(l, 12));
    or_gen_half_normal(m->L[l].Vc, n, seed, or_stream(l, 13));
  }
}

/* kcpu4.c:123-139: optional residual add, fp64 sum of squares in element order,
 * s = 1/sqrtf((float)(sum/D) + eps), xn = (h*s)*w. */
void or_rmsnorm(float* h, const float* y, int add, const float* w, float* xn, int D, float eps){
  double acc = 0.0;
  for(int e = 0; e < D; e++){
    const float xf = add ? h[e] + y[e] : h[e];
    h[e] = xf;
    acc += (double)xf * (double)xf;
  }
  const float s = 1.0f / sqrtf((float)(acc / D) + eps);
  for(int e = 0; e < D; e++){ const float t = h[e] * s; xn[e] = t * w[e]; }
}

/* kcpu4.c:223-236 with the rotary half rh = HD/2 (full-width NeoX rotary). */
void or_rope(const float* x, const float* cs, const float* sn, float* out, int HD){
  const int rh = HD / 2;
  for(int j = 0; j < rh; j++){
    const float a = x[j], b = x[j + rh];
    const float a0 = a * cs[j], b0 = b * sn[j], a1 = a * sn[j], b1 = b * cs[j];
    out[j] = a0 - b0;
    out[j + rh] = a1 + b1;
  }
}

static float or_silu(float x){ return x / (1.0f + expf(-x)); }

/* The score scale: the fp32 value nearest 1/sqrt(HD) (the reference's HD=256 uses 0.0625, which
 * is this value for 256). */
float or_attn_scale(int HD){ return (float)(1.0 / sqrt((double)HD)); }

/* Tree verification (not in the reference, which verifies linear chains only): the K/V row of
 * this token goes to cache slot `pos`, its rotary angle is that of position `rpos`, and it attends
 * to every slot below `tree_base` plus the slots tree_base + j whose bit j is set in `mask`
 * (its ancestors in the draft tree and itself). A plain decode step is pos == rpos with
 * tree_base = pos + 1. */
typedef struct { int rpos, tree_base; uint64_t mask[2]; } OTree;
static int or_attended(const OTree* tr, int t){
  if(t < tr->tree_base) return 1;
  const int j = t - tr->tree_base;
  return j < 128 && ((tr->mask[j >> 6] >> (j & 63)) & 1);
}

/* One attention block at position pos (kcpu4.c:218-285 without q/k norm and output gate). */
static void or_attn(OModel* m, OLayer* L, int pos, const OTree* tr){
  const OCfg* c = &m->c;
  const int NH = c->NH, NKV = c->NKV, HD = c->HD, G = NH / NKV, n = pos + 1, rh = HD / 2;
  or_matvec(&L->q, m->xn, m->q);
  or_matvec(&L->k, m->xn, m->k);
  or_matvec(&L->v, m->xn, m->v);
  const float* cs = m->cos_t + (size_t)tr->rpos * rh;
  const float* sn = m->sin_t + (size_t)tr->rpos * rh;
  for(int h = 0; h < NH; h++) or_rope(m->q + (size_t)h * HD, cs, sn, m->qr + (size_t)h * HD, HD);
  for(int kv = 0; kv < NKV; kv++){
    or_rope(m->k + (size_t)kv * HD, cs, sn, m->kr + (size_t)kv * HD, HD);
    uint16_t* K = L->Kc + ((size_t)pos * NKV + kv) * HD;
    uint16_t* V = L->Vc + ((size_t)pos * NKV + kv) * HD;
    for(int j = 0; j < HD; j++){ K[j] = or_f2h(m->kr[(size_t)kv * HD + j]); V[j] = or_f2h(m->v[(size_t)kv * HD + j]); }
  }
  const float scale = or_attn_scale(HD);
  #pragma omp parallel for schedule(static)
  for(int t = 0; t < n; t++){
    float kf[512];
    for(int kv = 0; kv < NKV; kv++){
      const uint16_t* K = L->Kc + ((size_t)t * NKV + kv) * HD;
      for(int j = 0; j < HD; j++) kf[j] = or_h2f(K[j]);
      for(int g = 0; g < G; g++){
        const float* q = m->qr + (size_t)(kv * G + g) * HD;
        float a = 0.f;
        for(int j = 0; j < HD; j++){ const float p = kf[j] * q[j]; a = a + p; }
        m->sc[(size_t)(kv * G + g) * c->ctx + t] = a * scale;
      }
    }
  }
  #pragma omp parallel for schedule(static)
  for(int hh = 0; hh < NH; hh++){
    float* s = m->sc + (size_t)hh * c->ctx;
    float mx = -1e30f;
    for(int t = 0; t < n; t++) if(or_attended(tr, t)) mx = fmaxf(mx, s[t]);
    float tot = 0.f;
    for(int t = 0; t < n; t++) if(or_attended(tr, t)) tot += expf(s[t] - mx);
    for(int t = 0; t < n; t++) s[t] = or_attended(tr, t) ? expf(s[t] - mx) / tot : 0.f;
  }
  #pragma omp parallel for schedule(static)
  for(int u = 0; u < NH * (HD / 32); u++){
    const int hh = u / (HD / 32), d0 = (u % (HD / 32)) * 32, kv = hh / G;
    const float* p = m->sc + (size_t)hh * c->ctx;
    float acc[32];
    for(int j = 0; j < 32; j++) acc[j] = 0.f;
    for(int t = 0; t < n; t++){
      const uint16_t* V = L->Vc + ((size_t)t * NKV + kv) * HD + d0;
      const float pt = p[t];
      for(int j = 0; j < 32; j++){ const float pv = pt * or_h2f(V[j]); acc[j] = acc[j] + pv; }
    }
    for(int j = 0; j < 32; j++) m->att[(size_t)hh * HD + d0 + j] = acc[j];
  }
  or_matvec(&L->o, m->att, m->y);
}

static void or_ffn(OModel* m, OLayer* L){
  or_rmsnorm(m->h, m->y, 1, L->ffn_norm, m->xn, m->c.D, m->c.eps);
  or_matvec(&L->gate, m->xn, m->g);
  or_matvec(&L->up, m->xn, m->u);
  for(int e = 0; e < m->c.NFF; e++) m->m[e] = or_silu(m->g[e]) * m->u[e];
  or_matvec(&L->down, m->m, m->y);
}

/* The MLP block of layer `layer` on M rows of x (row-major [M][D]) into y [M][D]: the steps of
 * ffn() (kcpu4.c:287-295) without the residual add -- xn = rmsnorm(x) * ffn_norm, gate and up
 * matvecs, silu(g) * u, the down matvec -- one row after another as the reference runs tokens.
 * Uses the model's scratch (h, xn, g, u, m); returns 0, or -3 on bad arguments. */
int or_ffn_block(OModel* m, int layer, const float* x, int M, float* y){
  if(layer < 0 || layer >= m->c.NL || M < 1) return -3;
  OLayer* L = m->L + layer;
  const int D = m->c.D;
  for(int r = 0; r < M; r++){
    memcpy(m->h, x + (size_t)r * D, (size_t)D * sizeof(float));
    or_rmsnorm(m->h, NULL, 0, L->ffn_norm, m->xn, D, m->c.eps);
    or_matvec(&L->gate, m->xn, m->g);
    or_matvec(&L->up, m->xn, m->u);
    for(int e = 0; e < m->c.NFF; e++) m->m[e] = or_silu(m->g[e]) * m->u[e];
    or_matvec(&L->down, m->m, y + (size_t)r * D);
  }
  return 0;
}

/* One token (kcpu4.c:303-335 structure). head != 0: logits into m->logits and the greedy id
 * (strict > scan, first index wins) is returned; head == 0 returns -1 and leaves h = residual. */
static int or_step_t(OModel* m, int tok, int pos, int head, const OTree* tr){
  const OCfg* c = &m->c;
  if(tok < 0 || tok >= c->vocab || pos < 0 || pos >= c->ctx || tr->rpos < 0 || tr->rpos >= c->ctx) return -3;
  or_dequant_row(&m->emb, tok, m->h);
  for(int l = 0; l < c->NL; l++){
    OLayer* L = m->L + l;
    or_rmsnorm(m->h, m->y, l > 0, L->attn_norm, m->xn, c->D, c->eps);
    or_attn(m, L, pos, tr);
    or_ffn(m, L);
  }
  if(!head){ for(int e = 0; e < c->D; e++) m->h[e] += m->y[e]; return -1; }
  or_rmsnorm(m->h, m->y, 1, m->out_norm, m->xn, c->D, c->eps);
  or_matvec(&m->out, m->xn, m->logits);
  int bi = 0; float bv = m->logits[0];
  for(int i = 1; i < c->vocab; i++) if(m->logits[i] > bv){ bv = m->logits[i]; bi = i; }
  return bi;
}

int or_step(OModel* m, int tok, int pos, int head){
  OTree tr = {pos, pos + 1, {0, 0}};
  return or_step_t(m, tok, pos, head, &tr);
}

/* Depths of the nodes of a draft tree given by parent pointers (parents[0] = -1, 0 <= parents[i]
 * < i); -1 if the tree is malformed. */
int or_tree_depths(const int* parents, int n, int* depth){
  if(n < 1 || n > 128 || parents[0] != -1) return -1;
  depth[0] = 0;
  for(int i = 1; i < n; i++){
    if(parents[i] < 0 || parents[i] >= i) return -1;
    depth[i] = depth[parents[i]] + 1;
  }
  return 0;
}

/* Verification pass over a draft tree of n nodes (node 0 is the last accepted token, at position
 * pos): node i is run as one decode step with K/V slot pos + i, rotary position pos + depth(i),
 * attending to the prefix [0, pos) and to its ancestors and itself. Logits of node i go to
 * logits[i * vocab]; returns 0, or -3 on bad arguments. Node order and arithmetic are those of
 * or_step, so a linear chain reproduces the greedy steps token for token. */
int or_verify(OModel* m, const int* tokens, const int* parents, int n, int pos, float* logits, int* best){
  int depth[128];
  if(or_tree_depths(parents, n, depth) || pos < 0 || pos + n > m->c.ctx) return -3;
  uint64_t anc[128][2];
  for(int i = 0; i < n; i++){
    anc[i][0] = anc[i][1] = 0;
    if(i > 0){ anc[i][0] = anc[parents[i]][0]; anc[i][1] = anc[parents[i]][1]; }
    anc[i][i >> 6] |= 1ull << (i & 63);
  }
  for(int i = 0; i < n; i++){
    OTree tr = {pos + depth[i], pos, {anc[i][0], anc[i][1]}};
    const int r = or_step_t(m, tokens[i], pos + i, 1, &tr);
    if(r < 0) return r;
    if(best) best[i] = r;
    if(logits) memcpy(logits + (size_t)i * m->c.vocab, m->logits, (size_t)m->c.vocab * sizeof(float));
  }
  return 0;
}

/* KV compaction after acceptance: the accepted path root = path[0] = 0, path[1..k] (node ids)
 * moves from slots pos + path[j] to positions pos + j, in increasing j (a node's id is at least
 * its depth, so no source is overwritten before it is read). */
int or_commit(OModel* m, const int* path, int k, int pos){
  const OCfg* c = &m->c;
  if(k < 0 || pos < 0) return -3;
  for(int j = 1; j <= k; j++) if(path[j] < j || pos + path[j] >= c->ctx) return -3;
  const size_t row = (size_t)c->NKV * c->HD;
  for(int l = 0; l < c->NL; l++)
    for(int j = 1; j <= k; j++){
      memmove(m->L[l].Kc + (size_t)(pos + j) * row, m->L[l].Kc + (size_t)(pos + path[j]) * row, row * 2);
      memmove(m->L[l].Vc + (size_t)(pos + j) * row, m->L[l].Vc + (size_t)(pos + path[j]) * row, row * 2);
    }
  return 0;
}

/* Accessors for ctypes callers. */
float* or_model_logits(OModel* m){ return m->logits; }
float* or_model_hidden(OModel* m){ return m->h; }
float* or_model_swiglu(OModel* m){ return m->m; }   /* SwiGLU output of the last layer run */
uint16_t* or_model_kcache(OModel* m, int layer){ return m->L[layer].Kc; }
uint16_t* or_model_vcache(OModel* m, int layer){ return m->L[layer].Vc; }
const uint8_t* or_model_tensor(OModel* m, int layer, int kind){
  if(layer < 0) return kind == OR_T_EMB ? m->emb.W : kind == OR_T_OUT ? m->out.W : NULL;
  OLayer* L = m->L + layer;
  switch(kind){
    case OR_T_Q: return L->q.W; case OR_T_K: return L->k.W; case OR_T_V: return L->v.W; case OR_T_O: return L->o.W;
    case OR_T_GATE: return L->gate.W; case OR_T_UP: return L->up.W; case OR_T_DOWN: return L->down.W;
    default: return NULL;
  }
}
int or_sizeof_cfg(void){ return (int)sizeof(OCfg); }
void or_set_threads(int n){
#ifdef _OPENMP
  if(n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
int or_get_threads(void){
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------------------------------------
 * Acceptance of a verified draft tree (speculative sampling), the deterministic rule the GPU
 * kernel k_accept (csrc/kq_accept.cuh) follows bit for bit.
 *
 * The reference accepts a deterministic draft (q one-hot) along a linear chain with numpy's RNG
 * (scripts/kindi_q4/kindi/spec.py:769-787, sampler spec.py:726-766, sampling.py:57-72); its
 * rng.choice is not reproducible on a GPU. This restatement generalises to a draft distribution
 * q per node and to trees, following speculative sampling (Leviathan et al. 2023; Chen et al.
 * 2023) and its multi-draft form with recursive rejection (SpecInfer, Miao et al. 2024):
 *   at node v with target p_v = softmax(z_v / T) and draft q_v = softmax(g_v) (the distribution
 *   v's children were drawn from), children c in increasing id:
 *     accept c  iff  u_acc[c] * q(d_c) < p(d_c)          (fp32)
 *     accepted: emit d_c, continue at c with p_c, q_c
 *     rejected: p <- max(0, p - q) / sum(max(0, p - q))  (back to p_v if that sum is 0)
 *   no child accepted (or a leaf): emit the inverse-CDF sample of p at u_fin[v], stop.
 *   T == 0 (greedy): accept c iff d_c is the argmax of z_v (lowest id on ties); emit the argmax
 *   of the last node.
 * Arithmetic (fp32, no contraction): e^t by kq_exp below; sums over the vocabulary are blocked:
 * blocks of 1024 consecutive ids (zero padded), each summed by a balanced pairwise tree, the
 * block sums added in block order; the inverse CDF walks the block sums in order, then the ids of
 * the chosen block sequentially from that prefix.
 * ------------------------------------------------------------------------------------------- */

/* e^t for t <= 0 (0 below -87): Cody-Waite reduction t = k ln2 + r with ln2 split in a high part
 * exact in fp32 and a low part, |r| <= ln2/2, then e^r by its Taylor series to degree 7 (Horner,
 * fused multiply-adds), scaled by 2^k. Error about 1 ulp; what matters is that the GPU kernel
 * computes the identical value. */
float or_kq_exp(float t){
  if(!(t >= -87.0f)) return 0.0f;
  /* fp32 constants: 1/ln2, ln2 = HI + LO (HI has 12 significant bits, so k * HI is exact), 1/n! */
  const float k = fmaf(t, 0x1.715476p+0f, 12582912.0f) - 12582912.0f;   /* round(t / ln2), 1.5 * 2^23 trick */
  float r = fmaf(-k, 0x1.62e4p-1f, t);
  r = fmaf(-k, 0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;            /* 1/5040 */
  p = fmaf(p, r, 0x1.6c16c2p-10f);      /* 1/720 */
  p = fmaf(p, r, 0x1.111112p-7f);       /* 1/120 */
  p = fmaf(p, r, 0x1.555556p-5f);       /* 1/24 */
  p = fmaf(p, r, 0x1.555556p-3f);       /* 1/6 */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  union { float f; int32_t i; } sc;
  sc.i = ((int32_t)k + 127) << 23;
  return p * sc.f;
}

#define OR_ABLK 1024
static float or_pairwise(const float* a, int n){
  if(n == 1) return a[0];
  return or_pairwise(a, n / 2) + or_pairwise(a + n / 2, n / 2);
}
/* Block sums into bs[] (ceil(V/1024) of them) and their in-order total. */
static float or_blocked_sum(const float* w, int V, float* bs){
  float buf[OR_ABLK];
  const int nb = (V + OR_ABLK - 1) / OR_ABLK;
  float tot = 0.0f;
  for(int b = 0; b < nb; b++){
    for(int i = 0; i < OR_ABLK; i++){ const int id = b * OR_ABLK + i; buf[i] = id < V ? w[id] : 0.0f; }
    bs[b] = or_pairwise(buf, OR_ABLK);
    tot = tot + bs[b];
  }
  return tot;
}
/* p = softmax(z * tau) with the rule above (tau = 1/T as the caller rounded it). */
static void or_softmax(const float* z, int V, float tau, float* p, float* bs){
  float mx = z[0];
  for(int i = 1; i < V; i++) if(z[i] > mx) mx = z[i];
  for(int i = 0; i < V; i++) p[i] = or_kq_exp((z[i] - mx) * tau);
  const float S = or_blocked_sum(p, V, bs);
  for(int i = 0; i < V; i++) p[i] = p[i] / S;
}
static int or_argmax(const float* z, int V){
  int bi = 0;
  for(int i = 1; i < V; i++) if(z[i] > z[bi]) bi = i;
  return bi;
}
static int or_inverse_cdf(const float* w, int V, float u, float* bs){
  const float W = or_blocked_sum(w, V, bs);
  const float target = u * W;
  const int nb = (V + OR_ABLK - 1) / OR_ABLK;
  float prefix = 0.0f;
  for(int b = 0; b < nb; b++){
    if(prefix + bs[b] > target){
      float run = prefix;
      for(int i = b * OR_ABLK; i < V && i < (b + 1) * OR_ABLK; i++){
        run = run + w[i];
        if(run > target) return i;
      }
    }
    prefix = prefix + bs[b];
  }
  for(int i = V - 1; i >= 0; i--) if(w[i] > 0.0f) return i;
  return 0;
}

/* Tree acceptance. z: target logits [n][V]; g: draft logits [n][V] (row v: the distribution of
 * v's children; unused for leaves and when tau == 0); tokens[c] the draft token of node c;
 * u_acc[c], u_fin[v] uniforms in [0,1). tau = 0: greedy. Writes the accepted node path
 * (path[0] = 0, then the accepted nodes) and the emitted tokens; returns the number of emitted
 * tokens (accepted drafts + 1), or -3 on bad arguments. */
int or_accept(const float* z, const float* g, const int* tokens, const int* parents, int n, int V, float tau,
              const float* u_acc, const float* u_fin, int* path, int* out){
  int depth[128];
  if(or_tree_depths(parents, n, depth)) return -3;
  float* p = (float*)malloc((size_t)V * sizeof(float));
  float* q = (float*)malloc((size_t)V * sizeof(float));
  float* bs = (float*)malloc((size_t)((V + OR_ABLK - 1) / OR_ABLK) * sizeof(float));
  int v = 0, np = 0, no = 0;
  path[np++] = 0;
  for(;;){
    const float* zv = z + (size_t)v * V;
    int acc = -1;
    if(tau == 0.0f){
      const int best = or_argmax(zv, V);
      for(int c = v + 1; c < n && acc < 0; c++) if(parents[c] == v && tokens[c] == best) acc = c;
      if(acc < 0){ out[no++] = best; break; }
    } else {
      or_softmax(zv, V, tau, p, bs);
      int first = 1;
      for(int c = v + 1; c < n && acc < 0; c++){
        if(parents[c] != v) continue;
        if(first){ or_softmax(g + (size_t)v * V, V, 1.0f, q, bs); first = 0; }
        const int d = tokens[c];
        if(u_acc[c] * q[d] < p[d]){ acc = c; break; }
        for(int i = 0; i < V; i++){ const float r = p[i] - q[i]; p[i] = r > 0.0f ? r : 0.0f; }
        const float R = or_blocked_sum(p, V, bs);
        if(R > 0.0f) for(int i = 0; i < V; i++) p[i] = p[i] / R;
        else or_softmax(zv, V, tau, p, bs);   /* empty residual (p == q): back to p_v */
      }
      if(acc < 0){ out[no++] = or_inverse_cdf(p, V, u_fin[v], bs); break; }
    }
    out[no++] = tokens[acc];
    path[np++] = acc;
    v = acc;
  }
  free(p); free(q); free(bs);
  return no;
}
