/*
 * CPU oracle for paged GQA decode attention.
 *
 * TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg use it as the checker / the timed CPU port.  The product
 * path never calls it.
 *
 * fp32 restatement of the reference's oracle, python/reference.py of
 * yuqiz7/mla-decode-kernels:
 *   gather_kv      (reference.py:7-18)  token t of request b lives in block
 *                  block_table[b, t / bs], slot t % bs;
 *   attention_ref  (reference.py:21-40) per (b, h), kv = h // (Hq // Hkv):
 *                  scores = (K[:, kv, :] @ q[b, h]) * scale;
 *                  w = softmax(scores); out[b, h] = w @ V[:, kv, :].
 * plus the online-softmax step and the split merge identity
 * (kernels/gqa_decode/v2_splitkv.cu:56-62, 97-107; docs/k1/notes_w1.md:74-95)
 * and the NHD element index (docs/k1/notes_w1.md:55-68).
 *
 * Parity is pinned against outputs of reference.py itself, stored in
 * tests/golden/ by tests/golden/make_golden.py.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HEAD_DIM 128

/* Minimal parallel-for over [0, n): worker threads pull indices from an
 * atomic counter. */
typedef void (*task_fn)(void* ctx, int64_t i);
typedef struct {
  task_fn fn;
  void* ctx;
  int64_t n;
  atomic_llong next;
} pfor_t;

static void* pfor_worker(void* arg) {
  pfor_t* pf = (pfor_t*)arg;
  for (;;) {
    const int64_t i = atomic_fetch_add(&pf->next, 1);
    if (i >= pf->n) break;
    pf->fn(pf->ctx, i);
  }
  return NULL;
}

static void parallel_for(int64_t n, int nthreads, task_fn fn, void* ctx) {
  pfor_t pf;
  pf.fn = fn;
  pf.ctx = ctx;
  pf.n = n;
  atomic_init(&pf.next, 0);
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if ((int64_t)nthreads > n) nthreads = (int)(n > 0 ? n : 1);
  pthread_t tids[256];
  int started = 0;
  for (int t = 1; t < nthreads; ++t)
    if (pthread_create(&tids[started], NULL, pfor_worker, &pf) == 0) ++started;
  pfor_worker(&pf);
  for (int t = 0; t < started; ++t) pthread_join(tids[t], NULL);
}

static inline float bf16_to_f32(uint16_t x) {
  const uint32_t u = (uint32_t)x << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* Element index of (block p, slot s, kv head h, dim j) in an NHD cache
 * [num_blocks, bs, Hkv, 128] (docs/k1/notes_w1.md:55-68). */
int64_t oracle_nhd_index(int64_t p, int64_t s, int64_t bs, int64_t Hkv, int64_t h, int64_t j) {
  return ((p * bs + s) * Hkv + h) * HEAD_DIM + j;
}

static inline float dot128(const uint16_t* krow, const float* qf) {
  float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int d = 0; d < HEAD_DIM; d += 8)
    for (int i = 0; i < 8; ++i) part[i] += bf16_to_f32(krow[d + i]) * qf[d + i];
  return ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
}

/* Per-(b, h) softmax pieces shared by the normalised and the state forms:
 * fills scores[0..S) with scale * (K q) and returns S. */
static int scores_bh(const uint16_t* q, const uint16_t* k, const int32_t* block_table,
                     const int32_t* seq_lens, int Hq, int Hkv, int bs, int max_blocks,
                     float scale, int64_t b, int h, float* qf, float** scores_out) {
  const int G = Hq / Hkv;
  const int kv = h / G;
  const int S = seq_lens[b] > 0 ? seq_lens[b] : 0;
  const uint16_t* qrow = q + ((size_t)b * Hq + h) * HEAD_DIM;
  for (int d = 0; d < HEAD_DIM; ++d) qf[d] = bf16_to_f32(qrow[d]);
  float* scores = (float*)malloc((size_t)(S > 0 ? S : 1) * sizeof(float));
  for (int t = 0; t < S; ++t) {
    const int64_t p = block_table[(size_t)b * max_blocks + t / bs];
    const uint16_t* krow = k + oracle_nhd_index(p, t % bs, bs, Hkv, kv, 0);
    scores[t] = dot128(krow, qf) * scale;
  }
  *scores_out = scores;
  return S;
}

typedef struct {
  const uint16_t *q, *k, *v;
  const int32_t *block_table, *seq_lens;
  int Hq, Hkv, bs, max_blocks;
  float scale;
  float *out, *m_out, *l_out, *acc_out;
} attn_ctx;

/* One (b, h) of attention_ref: normalised fp32 output row. */
static void attn_ref_task(void* vctx, int64_t bh) {
  const attn_ctx* c = (const attn_ctx*)vctx;
  const int64_t b = bh / c->Hq;
  const int h = (int)(bh % c->Hq);
  const int G = c->Hq / c->Hkv;
  float qf[HEAD_DIM];
  float* scores;
  const int S = scores_bh(c->q, c->k, c->block_table, c->seq_lens, c->Hq, c->Hkv, c->bs,
                          c->max_blocks, c->scale, b, h, qf, &scores);
  float o[HEAD_DIM];
  for (int d = 0; d < HEAD_DIM; ++d) o[d] = 0.f;
  if (S > 0) {
    float m = -INFINITY;
    for (int t = 0; t < S; ++t) m = scores[t] > m ? scores[t] : m;
    float sum = 0.f;
    for (int t = 0; t < S; ++t) {
      scores[t] = expf(scores[t] - m);
      sum += scores[t];
    }
    for (int t = 0; t < S; ++t) {
      const float w = scores[t] / sum;
      const int64_t p = c->block_table[(size_t)b * c->max_blocks + t / c->bs];
      const uint16_t* vrow = c->v + oracle_nhd_index(p, t % c->bs, c->bs, c->Hkv, h / G, 0);
      for (int d = 0; d < HEAD_DIM; ++d) o[d] += w * bf16_to_f32(vrow[d]);
    }
  }
  memcpy(c->out + bh * HEAD_DIM, o, sizeof o);
  free(scores);
}

/* One (b, h) of the unnormalised state form. */
static void attn_state_task(void* vctx, int64_t bh) {
  const attn_ctx* c = (const attn_ctx*)vctx;
  const int64_t b = bh / c->Hq;
  const int h = (int)(bh % c->Hq);
  const int G = c->Hq / c->Hkv;
  float qf[HEAD_DIM];
  float* scores;
  const int S = scores_bh(c->q, c->k, c->block_table, c->seq_lens, c->Hq, c->Hkv, c->bs,
                          c->max_blocks, c->scale, b, h, qf, &scores);
  float a[HEAD_DIM];
  for (int d = 0; d < HEAD_DIM; ++d) a[d] = 0.f;
  float m = -INFINITY, l = 0.f;
  for (int t = 0; t < S; ++t) m = scores[t] > m ? scores[t] : m;
  for (int t = 0; t < S; ++t) {
    const float e = expf(scores[t] - m);
    l += e;
    const int64_t p = c->block_table[(size_t)b * c->max_blocks + t / c->bs];
    const uint16_t* vrow = c->v + oracle_nhd_index(p, t % c->bs, c->bs, c->Hkv, h / G, 0);
    for (int d = 0; d < HEAD_DIM; ++d) a[d] += e * bf16_to_f32(vrow[d]);
  }
  c->m_out[bh] = m;
  c->l_out[bh] = l;
  memcpy(c->acc_out + bh * HEAD_DIM, a, sizeof a);
  free(scores);
}

/* attention_ref: out [B, Hq, 128] fp32, (b, h) pairs spread over nthreads.
 * A request with seq_len <= 0 gets zeros (what reference.py returns for an
 * empty softmax). */
void oracle_attention_ref(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          const int32_t* block_table, const int32_t* seq_lens, int B, int Hq,
                          int Hkv, int bs, int max_blocks, float scale, float* out,
                          int nthreads) {
  attn_ctx c = {q, k, v, block_table, seq_lens, Hq, Hkv, bs, max_blocks, scale,
                out, NULL, NULL, NULL};
  parallel_for((int64_t)B * Hq, nthreads, attn_ref_task, &c);
}

/* Unnormalised state per (b, h) in natural-log units: m = max_t s_t,
 * l = sum_t exp(s_t - m), acc = sum_t exp(s_t - m) V_t (s = scale * K q).
 * Empty requests: m = -inf, l = 0, acc = 0. */
void oracle_attention_state(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                            const int32_t* block_table, const int32_t* seq_lens, int B, int Hq,
                            int Hkv, int bs, int max_blocks, float scale, float* m_out,
                            float* l_out, float* acc_out, int nthreads) {
  attn_ctx c = {q, k, v, block_table, seq_lens, Hq, Hkv, bs, max_blocks, scale,
                NULL, m_out, l_out, acc_out};
  parallel_for((int64_t)B * Hq, nthreads, attn_state_task, &c);
}

/* One online-softmax pass over n scores with dv-wide values (the per-token
 * update of kernels/gqa_decode/v2_splitkv.cu:56-62), starting from the
 * neutral state.  Writes the unnormalised final state. */
void oracle_online_softmax(const float* scores, const float* values, int n, int dv, float* m_out,
                           float* l_out, float* acc_out) {
  float m = -INFINITY, l = 0.f;
  for (int j = 0; j < dv; ++j) acc_out[j] = 0.f;
  for (int t = 0; t < n; ++t) {
    const float mn = scores[t] > m ? scores[t] : m;
    const float alpha = expf(m - mn);
    const float p = expf(scores[t] - mn);
    l = l * alpha + p;
    for (int j = 0; j < dv; ++j) acc_out[j] = acc_out[j] * alpha + p * values[(size_t)t * dv + j];
    m = mn;
  }
  *m_out = m;
  *l_out = l;
}

/* Merge n unnormalised states (kernels/gqa_decode/v2_splitkv.cu:97-107):
 * M = max m_i, f_i = exp(m_i - M), L = sum l_i f_i, acc = sum acc_i f_i.
 * All-empty input (M = -inf) yields the neutral state. */
void oracle_merge_states(const float* m, const float* l, const float* acc, int n, int dv,
                         float* m_out, float* l_out, float* acc_out) {
  float M = -INFINITY;
  for (int i = 0; i < n; ++i) M = m[i] > M ? m[i] : M;
  for (int j = 0; j < dv; ++j) acc_out[j] = 0.f;
  float L = 0.f;
  if (M != -INFINITY) {
    for (int i = 0; i < n; ++i) {
      const float f = expf(m[i] - M);
      L += l[i] * f;
      for (int j = 0; j < dv; ++j) acc_out[j] += acc[(size_t)i * dv + j] * f;
    }
  }
  *m_out = M;
  *l_out = L;
}

/* ---- MLA absorbed-path decode (latent cache) -------------------------------
 *
 * The reference's roadmap kernel K2 (README.md "Roadmap": latent cache
 * [num_blocks, 64, 576], baseline FlashMLA) has no code in the reference
 * (kernels/mla_decode/ is empty), so this restates the operator FlashMLA's
 * tests check (flash_mla_with_kvcache against scaled dot-product attention on
 * the gathered cache; docs/k1/notes_w1.md:97-121 quotes its accounting):
 *   q [B, s_q, h_q, 576], one latent kv head: K = cache[t, 0:576],
 *   V = cache[t, 0:512];  for query position i, head h:
 *   scores_t = scale * q[b, i, h, :] . K_t over t < S_b
 *              (causal, s_q > 1: t < S_b - s_q + 1 + i),
 *   out[b, i, h, :] = softmax(scores) @ V,  lse[b, h, i] = ln sum_t exp(scores_t);
 * a query with no visible token gets out = 0 and lse = -inf.
 * Parity is unpinned against the reference (it has no implementation); the
 * tests cross-check this restatement against torch's fp32 SDPA. */

#define MLA_D 576
#define MLA_DV 512

typedef struct {
  const uint16_t *q, *kv;
  const int32_t *bt, *sl;
  int B, s_q, h_q, page, max_blocks, causal;
  float scale;
  float *out, *lse;
} mla_ctx_t;

static void mla_ref_task(void* vctx, int64_t row) {
  const mla_ctx_t* c = (const mla_ctx_t*)vctx;
  const int h = (int)(row % c->h_q);
  const int i = (int)((row / c->h_q) % c->s_q);
  const int b = (int)(row / ((int64_t)c->h_q * c->s_q));
  const int S = c->sl[b];
  int vis = c->causal ? S - c->s_q + 1 + i : S;
  if (vis > S) vis = S;
  if (vis < 0) vis = 0;
  float* o = c->out + row * MLA_DV;
  float* lse = c->lse + ((int64_t)b * c->h_q + h) * c->s_q + i;
  memset(o, 0, sizeof(float) * MLA_DV);
  if (vis == 0) {
    *lse = -INFINITY;
    return;
  }
  float qf[MLA_D];
  const uint16_t* qrow = c->q + row * MLA_D;
  for (int d = 0; d < MLA_D; ++d) qf[d] = bf16_to_f32(qrow[d]);
  float* sc = (float*)malloc(sizeof(float) * (size_t)vis);
  float mx = -INFINITY;
  for (int t = 0; t < vis; ++t) {
    const int p = c->bt[(int64_t)b * c->max_blocks + t / c->page];
    const uint16_t* krow = c->kv + ((int64_t)p * c->page + t % c->page) * MLA_D;
    float acc = 0.f;
    for (int d = 0; d < MLA_D; ++d) acc += bf16_to_f32(krow[d]) * qf[d];
    sc[t] = acc * c->scale;
    if (sc[t] > mx) mx = sc[t];
  }
  double sum = 0.0;
  for (int t = 0; t < vis; ++t) {
    sc[t] = expf(sc[t] - mx);
    sum += sc[t];
  }
  for (int t = 0; t < vis; ++t) {
    const int p = c->bt[(int64_t)b * c->max_blocks + t / c->page];
    const uint16_t* vrow = c->kv + ((int64_t)p * c->page + t % c->page) * MLA_D;
    const float w = (float)(sc[t] / sum);
    for (int d = 0; d < MLA_DV; ++d) o[d] += w * bf16_to_f32(vrow[d]);
  }
  *lse = (float)(log(sum) + mx);
  free(sc);
}

void oracle_mla_ref(const uint16_t* q, const uint16_t* kv, const int32_t* block_table,
                    const int32_t* seq_lens, int B, int s_q, int h_q, int page, int max_blocks,
                    float scale, int causal, float* out, float* lse, int nthreads) {
  mla_ctx_t c = {q, kv, block_table, seq_lens, B, s_q, h_q, page, max_blocks, causal, scale,
                 out, lse};
  parallel_for((int64_t)B * s_q * h_q, nthreads, mla_ref_task, &c);
}

/* ---- DSA-style sparse decode (K3): the indexer ------------------------------
 *
 * The reference's roadmap kernel K3 ("DSA-style sparse decode: indexer +
 * top-k + sparse gather", README.md "Roadmap") has no code in the reference.
 * Restated operator (DeepSeek sparse attention's lightning indexer): for
 * request b, query position i, cached token t < visible(b, i):
 *   I[b, i, t] = sum_j w[b, i, j] * relu(q_idx[b, i, j, :] . k_idx[t, :])
 * with H index heads of 128 dims, k_idx paged like the latent cache
 * ([num_blocks, page, 128]); tokens a query cannot see score -inf.  The
 * top-k selection and the attention over the selected tokens are restated
 * in oracle.py (selection) and oracle_mla_ref (attention). */

#define DSA_D 128

typedef struct {
  const uint16_t *q, *k;
  const float* w;
  const int32_t *bt, *sl;
  int B, s_q, H, page, max_blocks, causal, smax;
  float* scores;
} dsa_ctx_t;

static void dsa_scores_task(void* vctx, int64_t bi) {
  const dsa_ctx_t* c = (const dsa_ctx_t*)vctx;
  const int i = (int)(bi % c->s_q);
  const int b = (int)(bi / c->s_q);
  const int S = c->sl[b];
  int vis = c->causal ? S - c->s_q + 1 + i : S;
  if (vis > S) vis = S;
  if (vis < 0) vis = 0;
  float* out = c->scores + bi * c->smax;
  for (int t = 0; t < c->smax; ++t) out[t] = -INFINITY;
  float* qf = (float*)malloc(sizeof(float) * (size_t)c->H * DSA_D);
  const uint16_t* qrow = c->q + bi * c->H * DSA_D;
  for (int e = 0; e < c->H * DSA_D; ++e) qf[e] = bf16_to_f32(qrow[e]);
  const float* w = c->w + bi * c->H;
  for (int t = 0; t < vis && t < c->smax; ++t) {
    const int p = c->bt[(int64_t)b * c->max_blocks + t / c->page];
    const uint16_t* krow = c->k + ((int64_t)p * c->page + t % c->page) * DSA_D;
    float kf[DSA_D];
    for (int d = 0; d < DSA_D; ++d) kf[d] = bf16_to_f32(krow[d]);
    float s = 0.f;
    for (int j = 0; j < c->H; ++j) {
      float dot = 0.f;
      const float* qj = qf + j * DSA_D;
      for (int d = 0; d < DSA_D; ++d) dot += qj[d] * kf[d];
      s += w[j] * (dot > 0.f ? dot : 0.f);
    }
    out[t] = s;
  }
  free(qf);
}

void oracle_dsa_scores(const uint16_t* q_idx, const float* w_idx, const uint16_t* k_idx,
                       const int32_t* block_table, const int32_t* seq_lens, int B, int s_q, int H,
                       int page, int max_blocks, int causal, int smax, float* scores,
                       int nthreads) {
  dsa_ctx_t c = {q_idx, k_idx, w_idx, block_table, seq_lens, B, s_q, H, page, max_blocks, causal,
                 smax, scores};
  parallel_for((int64_t)B * s_q, nthreads, dsa_scores_task, &c);
}
