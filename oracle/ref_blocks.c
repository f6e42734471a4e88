/* ref_blocks.c -- TEST INFRASTRUCTURE ONLY (never part of the product): thin entry points into
 * the reference's own CPU engine, so that tests can check the oracle's blocks against it.
 *
 * The reference CPU engine keeps its block functions static: ffn (kcpu4.c:287-295) with rmsfold
 * (:123-139), fold (:89-93, an identity copy for these weights), gemv (:100-118) and q4_dot
 * (q4kernels.h:37-83). This file is compiled together with the unmodified reference source,
 * which it includes by the path given at build time (-DKCPU4_SOURCE, see oracle/Makefile), into
 * oracle/_ref/libkcpu4_blocks.so; nothing of the reference is copied here.
 *  - ref_ffn_block fills the reference's own Model / Layer structures with the caller's weights
 *    (Kindi pack layout) and runs its ffn once: y = down(silu(gate(xn)) * up(xn)),
 *    xn = rmsnorm(x + 0) * norm.
 *  - ref_head_step runs the reference's kc_step (:303-335) on a model of no layers: the embedding
 *    row of tok (q4_row), the final rmsfold with out_norm, the head GEMV and its argmax (strictly
 *    greater: the lowest index among equal logits).
 */
#include KCPU4_SOURCE
#include <stdlib.h>

static Mat ref_mat(const uint8_t* w, int R, int C, int type) {
  const int bs = type == 12 ? 144 : 210;
  Mat a;
  memset(&a, 0, sizeof a);
  a.W = w;
  a.S = NULL;
  a.R = R;
  a.C = C;
  a.type = type;
  a.offset = 0;
  a.bytes = (uint64_t)R * (uint64_t)(C / 256) * (uint64_t)bs;
  return a;
}

/* 0 on success, -1 when scratch could not be allocated. */
int ref_ffn_block(const uint8_t* wg, const uint8_t* wu, const uint8_t* wd, int tg, int tu, int td, int D, int NFF,
                  const float* norm, const float* x, float* y) {
  Model m;
  Layer L;
  memset(&m, 0, sizeof m);
  memset(&L, 0, sizeof L);
  const size_t big = (size_t)(NFF > D ? NFF : D);
  float* buf = (float*)calloc(3 * (size_t)D + big + 3 * (size_t)NFF, sizeof(float));
  if (!buf) return -1;
  m.D = D;
  m.NFF = NFF;
  m.L = &L;
  m.h = buf;
  m.y = m.h + D;
  m.xn = m.y + D;
  m.xp = m.xn + D;
  m.ffg = m.xp + big;
  m.ffu = m.ffg + NFF;
  m.m = m.ffu + NFF;
  L.post_norm = norm;
  L.ffg = ref_mat(wg, NFF, D, tg);
  L.ffu = ref_mat(wu, NFF, D, tu);
  L.ffd = ref_mat(wd, D, NFF, td);
  memcpy(m.h, x, sizeof(float) * (size_t)D);   /* m.y is zero: the residual add leaves x */
  ffn(&m, &L);
  memcpy(y, m.y, sizeof(float) * (size_t)D);
  free(buf);
  return 0;
}

/* The argmax token (and the logits [V]) of kc_step(tok, pos 0, head) on a model of no layers. */
int ref_head_step(const uint8_t* emb, int t_emb, const uint8_t* head, int t_head, int D, int V,
                  const float* out_norm, int tok, float* logits) {
  Model m;
  memset(&m, 0, sizeof m);
  float* buf = (float*)calloc(4 * (size_t)D + (size_t)V, sizeof(float));
  if (!buf) return -1;
  m.D = D;
  m.NL = 0;
  m.vocab = V;
  m.L = NULL;
  m.emb = ref_mat(emb, V, D, t_emb);
  m.head = ref_mat(head, V, D, t_head);
  m.out_norm = out_norm;
  m.h = buf;
  m.y = m.h + D;
  m.xn = m.y + D;
  m.xp = m.xn + D;
  m.logits = m.xp + D;
  const int best = kc_step(&m, tok, 0, 1);
  memcpy(logits, m.logits, sizeof(float) * (size_t)V);
  free(buf);
  return best;
}
