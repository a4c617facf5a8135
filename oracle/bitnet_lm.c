/*
 * CPU oracle of the BitNet ternary tag LM forward and greedy decode — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's baseline legs load this library, as the
 * checker of the B200 LM; the product never links it.
 *
 * Plain-C restatement of the reference's BitNet::forward (src/models/bitnet.hpp:376-440) with the
 * model dimensions as parameters (the reference fixes them at compile time,
 * src/models/bitnet_config.hpp:41-58), in the same operation order:
 *   h = embed[token]                                        (float)
 *   per layer (attention_block :490-585, ffn_block :589-617):
 *     x = rms_norm(h, attn_norm)                            (bitnet.hpp:234-250, double)
 *     q|k|v = bitlinear(w, x)                               (bitnet.hpp:447-471, exact integer)
 *     RoPE on q, k (GPT-NeoX halves, base 1e4)              (bitnet.hpp:472-488, double)
 *     causal softmax(q k^T / 8) v per head                  (double scores, float accumulation)
 *     h += bitlinear(wo, attn_out)
 *     x = rms_norm(h, ffn_norm); g, u = bitlinear(w_gate|w_up, x)
 *     h += bitlinear(w_down, float(silu(g) * u))            (double silu)
 *   logits = float(double dot(rms_norm(h, final_norm), embed[v]))   (tied lm_head, no quantisation)
 * Ternary weights are quantized once per row (quantize_weight_ternary is a pure function of the
 * row, so this equals the reference's per-call requantisation).
 * Greedy decode follows the reference's rule (src/infer/bitnet.hpp:282-318): argmax of the last
 * position's logits, ties to the smallest id, stop before <eos> (id 2) or at max_len tokens.  The
 * decode keeps a per-position K/V cache: every quantity of a position depends only on that
 * position and the earlier ones, so this equals recomputing the whole prefix each step.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

float oracle_quantize_weight_ternary(const float* w, size_t n, int8_t* q);
float oracle_quantize_activation_int8(const float* x, size_t n, int8_t* q);

typedef struct {
  int vocab, d_model, n_layers, n_heads, ffn_dim, max_seq;
  double rope_base, rms_eps;
  int per_tensor_scale; /* 0: alpha per output row (the reference); 1: one alpha per tensor */
} lm_config;

typedef struct {
  const float *attn_norm, *wq, *wk, *wv, *wo, *ffn_norm, *w_gate, *w_up, *w_down;
} lm_layer_f32;

/* quantized linear: q [N, K] int8 in {-1, 0, 1}, alpha [N] */
typedef struct {
  int N, K;
  int8_t* q;
  float* alpha;
} tlin;

typedef struct {
  lm_config c;
  const float* embed;
  const float* final_norm;
  const float** attn_norm;
  const float** ffn_norm;
  tlin *wq, *wk, *wv, *wo, *wg, *wu, *wd;
} lm_model;

static void tlin_init(tlin* t, const float* w, int N, int K, int per_tensor) {
  t->N = N;
  t->K = K;
  t->q = (int8_t*)malloc((size_t)N * K);
  t->alpha = (float*)malloc(sizeof(float) * N);
  if (!per_tensor) {
    for (int n = 0; n < N; ++n)
      t->alpha[n] = oracle_quantize_weight_ternary(w + (size_t)n * K, (size_t)K, t->q + (size_t)n * K);
    return;
  }
  /* the same absmean rule over the whole tensor (row-major order) */
  oracle_quantize_weight_ternary(w, (size_t)N * K, t->q);
  double sum_abs = 0.0;
  for (size_t i = 0; i < (size_t)N * K; ++i) sum_abs += fabs((double)w[i]);
  const float a = (float)(sum_abs / (double)((size_t)N * K));
  for (int n = 0; n < N; ++n) t->alpha[n] = a;
}

static void tlin_free(tlin* t) {
  free(t->q);
  free(t->alpha);
}

/* y[N] = bitlinear(x[K]) with the pre-quantized weights (bitnet.hpp:447-471) */
static void tlin_apply(const tlin* t, const float* x, float* y, int8_t* xq) {
  const float xs = oracle_quantize_activation_int8(x, (size_t)t->K, xq);
  for (int n = 0; n < t->N; ++n) {
    const int8_t* wr = t->q + (size_t)n * t->K;
    long long acc = 0;
    for (int i = 0; i < t->K; ++i) acc += (long long)wr[i] * (long long)xq[i];
    y[n] = (float)((double)acc * (double)t->alpha[n] * (double)xs);
  }
}

/* rms_norm (bitnet.hpp:234-250) */
static void rms_norm(const float* x, const float* w, float* out, int n, double eps) {
  double ms = 0.0;
  for (int i = 0; i < n; ++i) {
    const double v = (double)x[i];
    ms += v * v;
  }
  ms /= (double)n;
  const double inv = 1.0 / sqrt(ms + eps);
  for (int i = 0; i < n; ++i) out[i] = (float)((double)x[i] * inv * (double)w[i]);
}

/* RoPE (bitnet.hpp:472-488) */
static void apply_rope(float* vec, int pos, int head_dim, double base) {
  const int half = head_dim / 2;
  for (int i = 0; i < half; ++i) {
    const double freq = 1.0 / pow(base, (double)(2 * i) / (double)head_dim);
    const double angle = (double)pos * freq;
    const double cs = cos(angle);
    const double sn = sin(angle);
    const double a = (double)vec[i];
    const double b = (double)vec[i + half];
    vec[i] = (float)(a * cs - b * sn);
    vec[i + half] = (float)(a * sn + b * cs);
  }
}

void* oracle_lm_create(const lm_config* c, const float* embed, const float* final_norm,
                       const lm_layer_f32* layers) {
  lm_model* m = (lm_model*)calloc(1, sizeof(lm_model));
  m->c = *c;
  m->embed = embed;
  m->final_norm = final_norm;
  const int L = c->n_layers, D = c->d_model, F = c->ffn_dim;
  m->attn_norm = (const float**)malloc(sizeof(float*) * L);
  m->ffn_norm = (const float**)malloc(sizeof(float*) * L);
  tlin** lists[7] = {&m->wq, &m->wk, &m->wv, &m->wo, &m->wg, &m->wu, &m->wd};
  for (int k = 0; k < 7; ++k) *lists[k] = (tlin*)malloc(sizeof(tlin) * L);
  for (int l = 0; l < L; ++l) {
    m->attn_norm[l] = layers[l].attn_norm;
    m->ffn_norm[l] = layers[l].ffn_norm;
    const int pt = c->per_tensor_scale;
    tlin_init(&m->wq[l], layers[l].wq, D, D, pt);
    tlin_init(&m->wk[l], layers[l].wk, D, D, pt);
    tlin_init(&m->wv[l], layers[l].wv, D, D, pt);
    tlin_init(&m->wo[l], layers[l].wo, D, D, pt);
    tlin_init(&m->wg[l], layers[l].w_gate, F, D, pt);
    tlin_init(&m->wu[l], layers[l].w_up, F, D, pt);
    tlin_init(&m->wd[l], layers[l].w_down, D, F, pt);
  }
  return m;
}

void oracle_lm_destroy(void* p) {
  lm_model* m = (lm_model*)p;
  if (!m) return;
  for (int l = 0; l < m->c.n_layers; ++l) {
    tlin_free(&m->wq[l]);
    tlin_free(&m->wk[l]);
    tlin_free(&m->wv[l]);
    tlin_free(&m->wo[l]);
    tlin_free(&m->wg[l]);
    tlin_free(&m->wu[l]);
    tlin_free(&m->wd[l]);
  }
  free(m->wq);
  free(m->wk);
  free(m->wv);
  free(m->wo);
  free(m->wg);
  free(m->wu);
  free(m->wd);
  free(m->attn_norm);
  free(m->ffn_norm);
  free(m);
}

/* Decode state of one sequence: K/V cache [L][max_seq][D] (K after RoPE). */
typedef struct {
  float *K, *V;
  int len;
} lm_state;

/* Runs position `pos` (= st->len) with token `tok` through every layer, appends its K/V, and
 * writes the logits of this position when `logits` is not NULL. */
static void step(const lm_model* m, lm_state* st, int tok, float* logits) {
  const lm_config* c = &m->c;
  const int D = c->d_model, F = c->ffn_dim, H = c->n_heads, hd = D / H;
  const int pos = st->len;
  float* h = (float*)malloc(sizeof(float) * D);
  float* x = (float*)malloc(sizeof(float) * D);
  float* q = (float*)malloc(sizeof(float) * D);
  float* ao = (float*)malloc(sizeof(float) * D);
  float* pr = (float*)malloc(sizeof(float) * D);
  float* g = (float*)malloc(sizeof(float) * F);
  float* u = (float*)malloc(sizeof(float) * F);
  float* inter = (float*)malloc(sizeof(float) * F);
  int8_t* xq = (int8_t*)malloc((size_t)(F > D ? F : D));
  double* scores = (double*)malloc(sizeof(double) * (pos + 1));
  memcpy(h, m->embed + (size_t)tok * D, sizeof(float) * D);
  const double scale = 1.0 / sqrt((double)hd);
  for (int l = 0; l < c->n_layers; ++l) {
    float* Kl = st->K + ((size_t)l * c->max_seq) * D;
    float* Vl = st->V + ((size_t)l * c->max_seq) * D;
    rms_norm(h, m->attn_norm[l], x, D, c->rms_eps);
    tlin_apply(&m->wq[l], x, q, xq);
    tlin_apply(&m->wk[l], x, Kl + (size_t)pos * D, xq);
    tlin_apply(&m->wv[l], x, Vl + (size_t)pos * D, xq);
    for (int a = 0; a < H; ++a) {
      apply_rope(q + a * hd, pos, hd, c->rope_base);
      apply_rope(Kl + (size_t)pos * D + a * hd, pos, hd, c->rope_base);
    }
    for (int i = 0; i < D; ++i) ao[i] = 0.0f;
    for (int a = 0; a < H; ++a) {
      const int off = a * hd;
      double maxv = -1e300;
      for (int j = 0; j <= pos; ++j) {
        const float* kj = Kl + (size_t)j * D + off;
        double dot = 0.0;
        for (int d = 0; d < hd; ++d) dot += (double)q[off + d] * (double)kj[d];
        dot *= scale;
        scores[j] = dot;
        if (dot > maxv) maxv = dot;
      }
      double sum = 0.0;
      for (int j = 0; j <= pos; ++j) {
        const double e = exp(scores[j] - maxv);
        scores[j] = e;
        sum += e;
      }
      const double inv = 1.0 / sum;
      for (int j = 0; j <= pos; ++j) {
        const double w = scores[j] * inv;
        const float* vj = Vl + (size_t)j * D + off;
        for (int d = 0; d < hd; ++d) ao[off + d] += (float)(w * (double)vj[d]);
      }
    }
    tlin_apply(&m->wo[l], ao, pr, xq);
    for (int i = 0; i < D; ++i) h[i] += pr[i];
    rms_norm(h, m->ffn_norm[l], x, D, c->rms_eps);
    tlin_apply(&m->wg[l], x, g, xq);
    tlin_apply(&m->wu[l], x, u, xq);
    for (int f = 0; f < F; ++f) {
      const double gv = (double)g[f];
      const double silu = gv / (1.0 + exp(-gv));
      inter[f] = (float)(silu * (double)u[f]);
    }
    tlin_apply(&m->wd[l], inter, pr, xq);
    for (int i = 0; i < D; ++i) h[i] += pr[i];
  }
  st->len = pos + 1;
  if (logits) {
    rms_norm(h, m->final_norm, x, D, c->rms_eps);
    for (int v = 0; v < c->vocab; ++v) {
      const float* wv = m->embed + (size_t)v * D;
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc += (double)x[d] * (double)wv[d];
      logits[v] = (float)acc;
    }
  }
  free(h);
  free(x);
  free(q);
  free(ao);
  free(pr);
  free(g);
  free(u);
  free(inter);
  free(xq);
  free(scores);
}

static void state_init(const lm_model* m, lm_state* st) {
  const size_t n = (size_t)m->c.n_layers * m->c.max_seq * m->c.d_model;
  st->K = (float*)calloc(n, sizeof(float));
  st->V = (float*)calloc(n, sizeof(float));
  st->len = 0;
}

static void state_free(lm_state* st) {
  free(st->K);
  free(st->V);
}

/* Logits of every position of tokens[S] (BitNet::forward): logits [S, vocab].  Returns 0, or -1
 * when S is outside [1, max_seq] or a token is out of range. */
int oracle_lm_forward(void* p, const int* tokens, int S, float* logits) {
  const lm_model* m = (const lm_model*)p;
  if (S <= 0 || S > m->c.max_seq) return -1;
  for (int s = 0; s < S; ++s)
    if (tokens[s] < 0 || tokens[s] >= m->c.vocab) return -1;
  lm_state st;
  state_init(m, &st);
  for (int s = 0; s < S; ++s) step(m, &st, tokens[s], logits + (size_t)s * m->c.vocab);
  state_free(&st);
  return 0;
}

/* Greedy decode of one prompt (src/infer/bitnet.hpp:282-318 rule): writes the generated ids
 * (without <eos>) to out and returns their count, or -1 on invalid input. */
int oracle_lm_generate(void* p, const int* prompt, int P, int max_len, int eos, int* out) {
  const lm_model* m = (const lm_model*)p;
  if (P <= 0 || P > max_len || max_len > m->c.max_seq) return -1;
  for (int s = 0; s < P; ++s)
    if (prompt[s] < 0 || prompt[s] >= m->c.vocab) return -1;
  lm_state st;
  state_init(m, &st);
  float* logits = (float*)malloc(sizeof(float) * m->c.vocab);
  for (int s = 0; s < P; ++s) step(m, &st, prompt[s], s == P - 1 ? logits : NULL);
  int n = 0, seq_len = P;
  while (seq_len < max_len) {
    int best = 0;
    float bestv = logits[0];
    for (int v = 1; v < m->c.vocab; ++v)
      if (logits[v] > bestv) {
        bestv = logits[v];
        best = v;
      }
    if (best == eos) break;
    out[n++] = best;
    ++seq_len;
    if (seq_len < max_len) step(m, &st, best, logits);
  }
  free(logits);
  state_free(&st);
  return n;
}
