/* CPU oracle for the KV-cached Shahd decode path — TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * f64 restatement of the reference's TypeScript; each function cites the reference file:line it
 * follows. Under Compute.Precision "F32" every TENSOR buffer of the reference is a Float32Array, so
 * each store into a tensor rounds to f32 (ST() below), while the cached row math keeps f64 scratch and
 * an f64 KV cache (Brain/Sampling/CachedRowMath.ts:4-5, KvCache.ts:14-15). */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static __thread char g_err[512];

static int Fail(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return -1;
}

const char* oracle_last_error(void) { return g_err; }

/* ------------------------------------------------------------------------------------------------
 * Brain/Random/SeededRng.ts
 * ---------------------------------------------------------------------------------------------- */

/* MixSeed, SeededRng.ts:7-12 (Math.imul = low 32 bits of the product). */
uint32_t oracle_mix_seed(uint32_t seed, uint32_t stream) {
  uint32_t x = seed ^ (uint32_t)((stream + 1u) * 0x9e3779b9u);
  x = (x ^ (x >> 16)) * 0x45d9f3bu;
  x = (x ^ (x >> 16)) * 0x45d9f3bu;
  return x ^ (x >> 16);
}

/* NextUint32, SeededRng.ts:32-35. */
uint32_t oracle_rng_next_u32(uint32_t* state) {
  *state = *state * 1664525u + 1013904223u;
  return *state;
}

/* NextFloat, SeededRng.ts:38-40. */
double oracle_rng_next_float(uint32_t* state) { return (double)oracle_rng_next_u32(state) / 4294967296.0; }

/* NextGaussian, SeededRng.ts:43-47: Box-Muller with the 1e-12 guard; (2*PI)*V evaluated left to right. */
double oracle_rng_next_gaussian(uint32_t* state) {
  double u = oracle_rng_next_float(state);
  double v = oracle_rng_next_float(state);
  return sqrt(-2.0 * log(u + 1e-12)) * cos(2.0 * M_PI * v);
}

/* CreateRngStreams, SeededRng.ts:58-65: Init, Data, Dropout, Sampling. */
void oracle_create_streams(uint32_t seed, uint32_t out_states[4]) {
  for (uint32_t i = 0; i < 4; i++) out_states[i] = oracle_mix_seed(seed, i);
}

/* ------------------------------------------------------------------------------------------------
 * Parameter layout: Shahd.Parameters() (Shahd.ts:87-94) = Embedding [Wte, Wpe?] (Embedding.ts:28-30),
 * per block [Ln1 gamma, beta?] + Attn [Wq..., Wk..., Wv..., Wo...] (MultiHeadAttention.ts:76-78)
 * + [Ln2 ...] + Mlp [Wfc, Bfc, Wproj, Bproj | W1, W3, W2] (Mlp.ts:59-65), LnFinal, LmHead?, LmHeadBias.
 * ---------------------------------------------------------------------------------------------- */

typedef struct LayerOff {
  int64_t ln1_g, ln1_b, ln2_g, ln2_b;
  int64_t wq, wk, wv, wo; /* first head; heads are contiguous, [E,d] / [d,E] each */
  int64_t wfc, bfc, wproj, bproj, w1, w3, w2;
} LayerOff;

typedef struct Layout {
  int64_t wte, wpe, lnf_g, lnf_b, lm_head, lm_bias, total;
  LayerOff* layers;
} Layout;

static int CheckCfg(const OracleCfg* c) {
  if (c->embed_dim < 1 || c->num_layers < 1 || c->num_heads < 1 || c->kv_heads < 1 || c->block_size < 1 ||
      c->vocab_size < 1 || c->mlp_hidden < 1)
    return Fail("oracle: non-positive model dimension");
  if (c->embed_dim % c->num_heads != 0) return Fail("oracle: EmbedDim %d not divisible by NumHeads %d", c->embed_dim, c->num_heads);
  if (c->num_heads % c->kv_heads != 0) return Fail("oracle: NumHeads %d not divisible by KvHeads %d", c->num_heads, c->kv_heads);
  int d = c->embed_dim / c->num_heads;
  if (c->position_scheme == 1 && d % 2 != 0) return Fail("oracle: RoPE needs an even head dim, got %d", d);
  return 0;
}

static int64_t BuildLayout(const OracleCfg* c, Layout* lay) {
  const int64_t E = c->embed_dim, H = c->num_heads, Hk = c->kv_heads, d = E / H, F = c->mlp_hidden;
  const int ln = c->norm_kind == 0;
  int64_t o = 0;
  lay->wte = o; o += (int64_t)c->vocab_size * E;
  lay->wpe = -1;
  if (c->position_scheme == 0) { lay->wpe = o; o += (int64_t)c->block_size * E; }
  lay->layers = (LayerOff*)calloc((size_t)c->num_layers, sizeof(LayerOff));
  for (int l = 0; l < c->num_layers; l++) {
    LayerOff* L = &lay->layers[l];
    L->ln1_g = o; o += E;
    L->ln1_b = -1; if (ln) { L->ln1_b = o; o += E; }
    L->wq = o; o += H * E * d;
    L->wk = o; o += Hk * E * d;
    L->wv = o; o += Hk * E * d;
    L->wo = o; o += H * d * E;
    L->ln2_g = o; o += E;
    L->ln2_b = -1; if (ln) { L->ln2_b = o; o += E; }
    L->wfc = L->bfc = L->wproj = L->bproj = L->w1 = L->w3 = L->w2 = -1;
    if (c->mlp_kind == 0) {
      L->wfc = o; o += E * F;
      L->bfc = o; o += F;
      L->wproj = o; o += F * E;
      L->bproj = o; o += E;
    } else {
      L->w1 = o; o += E * F;
      L->w3 = o; o += E * F;
      L->w2 = o; o += F * E;
    }
  }
  lay->lnf_g = o; o += E;
  lay->lnf_b = -1; if (ln) { lay->lnf_b = o; o += E; }
  lay->lm_head = -1;
  if (!c->weight_tying) { lay->lm_head = o; o += E * c->vocab_size; }
  lay->lm_bias = o; o += c->vocab_size;
  lay->total = o;
  return o;
}

int64_t oracle_param_count(const OracleCfg* cfg) {
  if (CheckCfg(cfg)) return -1;
  Layout lay;
  int64_t n = BuildLayout(cfg, &lay);
  free(lay.layers);
  return n;
}

static double StoreF32(double x) { return (double)(float)x; }

/* RandN (TensorFactories.ts:23-30) through InitWeight (InitPolicy.ts:15-24). */
static void RandN(double* dst, int64_t count, double scale, uint32_t* rng, int f32) {
  for (int64_t i = 0; i < count; i++) {
    double v = oracle_rng_next_gaussian(rng) * scale;
    dst[i] = f32 ? StoreF32(v) : v;
  }
}

static void Fill(double* dst, int64_t count, double v) {
  for (int64_t i = 0; i < count; i++) dst[i] = v;
}

/* Construction order: Shahd.ts:30-39 → Embedding.ts:14-18 (Wte, Wpe) → per Block (Block.ts:16-22):
 * NormLayer (Filled 1 / Zeros, NormLayer.ts:15-20), MultiHeadAttention.ts:36-43 (Wq_h, Wo_h per head,
 * then Wk, Wv per KV head), NormLayer, Mlp.ts:26-40 → LnFinal → LmHead (untied) → LmHeadBias zeros. */
int oracle_init_params(const OracleCfg* c, uint32_t seed, double* p) {
  if (CheckCfg(c)) return -1;
  Layout lay;
  BuildLayout(c, &lay);
  memset(p, 0, sizeof(double) * (size_t)lay.total);
  uint32_t streams[4];
  oracle_create_streams(seed, streams);
  uint32_t rng = streams[0];
  const int64_t E = c->embed_dim, H = c->num_heads, Hk = c->kv_heads, d = E / H, F = c->mlp_hidden;
  const double s0 = c->init_scale;
  const double sres = c->use_scaled_residual_init ? c->init_scale / sqrt(2.0 * c->num_layers) : c->init_scale;
  const int f32 = c->precision_f32;
  RandN(p + lay.wte, (int64_t)c->vocab_size * E, s0, &rng, f32);
  if (lay.wpe >= 0) RandN(p + lay.wpe, (int64_t)c->block_size * E, s0, &rng, f32);
  for (int l = 0; l < c->num_layers; l++) {
    LayerOff* L = &lay.layers[l];
    Fill(p + L->ln1_g, E, 1.0);
    for (int64_t h = 0; h < H; h++) {
      RandN(p + L->wq + h * E * d, E * d, s0, &rng, f32);
      RandN(p + L->wo + h * d * E, d * E, sres, &rng, f32);
    }
    for (int64_t g = 0; g < Hk; g++) {
      RandN(p + L->wk + g * E * d, E * d, s0, &rng, f32);
      RandN(p + L->wv + g * E * d, E * d, s0, &rng, f32);
    }
    Fill(p + L->ln2_g, E, 1.0);
    if (c->mlp_kind == 0) {
      RandN(p + L->wfc, E * F, s0, &rng, f32);
      RandN(p + L->wproj, F * E, sres, &rng, f32);
    } else {
      RandN(p + L->w1, E * F, s0, &rng, f32);
      RandN(p + L->w3, E * F, s0, &rng, f32);
      RandN(p + L->w2, F * E, sres, &rng, f32);
    }
  }
  Fill(p + lay.lnf_g, E, 1.0);
  if (lay.lm_head >= 0) RandN(p + lay.lm_head, E * c->vocab_size, s0, &rng, f32);
  free(lay.layers);
  return 0;
}

/* ------------------------------------------------------------------------------------------------
 * Seam matmuls
 * ---------------------------------------------------------------------------------------------- */

/* TsBackend.MatMul (Brain/ComputeBackend/TsBackend.ts): ikj with the zero skip, out overwritten. */
void oracle_matmul(const double* a, const double* b, double* out, int m, int k, int n) {
  memset(out, 0, sizeof(double) * (size_t)m * n);
  for (int i = 0; i < m; i++)
    for (int p = 0; p < k; p++) {
      double av = a[(size_t)i * k + p];
      if (av == 0) continue;
      const double* br = b + (size_t)p * n;
      double* o = out + (size_t)i * n;
      for (int j = 0; j < n; j++) o[j] += av * br[j];
    }
}

/* MatMulNtInto / MatMulNtAcc semantics (ComputeBackend.ts:23-42; TsBackend.MatMulNtInto): p-ascending
 * dot from zero, then overwrite or add. */
void oracle_matmul_nt(const double* a, const double* bt, double* out, int m, int k, int n, int acc) {
  for (int i = 0; i < m; i++)
    for (int j = 0; j < n; j++) {
      double s = 0;
      for (int p = 0; p < k; p++) s += a[(size_t)i * k + p] * bt[(size_t)j * k + p];
      if (acc) out[(size_t)i * n + j] += s;
      else out[(size_t)i * n + j] = s;
    }
}

/* MatMulTnAcc semantics (ComputeBackend.ts:38-41): db[K,N] (+)= aᵀ @ dout, i ascending. */
void oracle_matmul_tn(const double* a, const double* dout, double* db, int m, int k, int n, int acc) {
  for (int p = 0; p < k; p++) {
    double* row = db + (size_t)p * n;
    if (!acc)
      for (int j = 0; j < n; j++) row[j] = 0;
    for (int i = 0; i < m; i++) {
      double av = a[(size_t)i * k + p];
      for (int j = 0; j < n; j++) row[j] += av * dout[(size_t)i * n + j];
    }
  }
}

/* ------------------------------------------------------------------------------------------------
 * Model
 * ---------------------------------------------------------------------------------------------- */

struct OracleModel {
  OracleCfg cfg;
  Layout lay;
  double* p;
  int E, L, H, Hk, d, F, C, V, G;
  double scale; /* Derived.AttentionScale = 1/sqrt(HeadDim), DeriveConfig.ts:15 */
  double* freq; /* RopeFrequencies, RotaryEmbedding.ts:17-22 */
};

struct OracleCache {
  int L, Hk, d, C;
  double* keys;
  double* values;
  int* lengths;
};

OracleModel* oracle_model_create(const OracleCfg* cfg, const double* params) {
  if (CheckCfg(cfg)) return NULL;
  OracleModel* m = (OracleModel*)calloc(1, sizeof(OracleModel));
  m->cfg = *cfg;
  BuildLayout(cfg, &m->lay);
  m->p = (double*)malloc(sizeof(double) * (size_t)m->lay.total);
  memcpy(m->p, params, sizeof(double) * (size_t)m->lay.total);
  m->E = cfg->embed_dim; m->L = cfg->num_layers; m->H = cfg->num_heads; m->Hk = cfg->kv_heads;
  m->d = m->E / m->H; m->F = cfg->mlp_hidden; m->C = cfg->block_size; m->V = cfg->vocab_size;
  m->G = m->H / m->Hk;
  m->scale = 1.0 / sqrt((double)m->d);
  m->freq = (double*)malloc(sizeof(double) * (size_t)(m->d / 2 + 1));
  for (int i = 0; i < m->d / 2; i++) m->freq[i] = pow(10000.0, (-2.0 * i) / m->d);
  return m;
}

void oracle_model_destroy(OracleModel* m) {
  if (!m) return;
  free(m->lay.layers);
  free(m->p);
  free(m->freq);
  free(m);
}

/* KvCache (Brain/Sampling/KvCache.ts:20-49): one f64 [Capacity, HeadDim] slot per (layer, KV head). */
OracleCache* oracle_cache_create(const OracleModel* m) {
  OracleCache* c = (OracleCache*)calloc(1, sizeof(OracleCache));
  c->L = m->L; c->Hk = m->Hk; c->d = m->d; c->C = m->C;
  size_t n = (size_t)c->L * c->Hk * c->C * c->d;
  c->keys = (double*)calloc(n, sizeof(double));
  c->values = (double*)calloc(n, sizeof(double));
  c->lengths = (int*)calloc((size_t)c->L * c->Hk, sizeof(int));
  return c;
}

void oracle_cache_destroy(OracleCache* c) {
  if (!c) return;
  free(c->keys); free(c->values); free(c->lengths); free(c);
}

/* KvCache.Length, KvCache.ts:52-54: the last slot's count. */
int oracle_cache_length(const OracleCache* c) { return c->lengths[c->L * c->Hk - 1]; }

static void CacheReset(OracleCache* c) { memset(c->lengths, 0, sizeof(int) * (size_t)c->L * c->Hk); }

/* KvCache.AppendRows, KvCache.ts:70-88. */
static int CacheAppendRows(OracleCache* c, int layer, int g, const double* k, const double* v, int rows) {
  int idx = layer * c->Hk + g;
  int pos = c->lengths[idx];
  if (pos + rows > c->C) return Fail("KvCache.AppendRows: %d+%d tokens exceed capacity %d", pos, rows, c->C);
  size_t base = (size_t)idx * c->C * c->d + (size_t)pos * c->d;
  memcpy(c->keys + base, k, sizeof(double) * (size_t)rows * c->d);
  memcpy(c->values + base, v, sizeof(double) * (size_t)rows * c->d);
  c->lengths[idx] = pos + rows;
  return 0;
}

int oracle_cache_read(const OracleCache* c, int layer, int g, double* k_out, double* v_out) {
  if (layer < 0 || layer >= c->L || g < 0 || g >= c->Hk) return Fail("KvCache: (layer %d, kv head %d) outside", layer, g);
  int idx = layer * c->Hk + g;
  size_t base = (size_t)idx * c->C * c->d;
  size_t n = (size_t)c->lengths[idx] * c->d;
  if (k_out) memcpy(k_out, c->keys + base, n * sizeof(double));
  if (v_out) memcpy(v_out, c->values + base, n * sizeof(double));
  return c->lengths[idx];
}

/* ------------------------------------------------------------------------------------------------
 * Row math: Brain/Sampling/CachedRowMath.ts
 * ---------------------------------------------------------------------------------------------- */

/* MatMulRow, CachedRowMath.ts:14-23: X[K] @ W[K,N], k ascending, zero skip. */
static void MatMulRow(const double* x, const double* w, int K, int N, double* out) {
  for (int n = 0; n < N; n++) out[n] = 0;
  for (int k = 0; k < K; k++) {
    double xk = x[k];
    if (xk == 0) continue;
    const double* wr = w + (size_t)k * N;
    for (int n = 0; n < N; n++) out[n] += xk * wr[n];
  }
}

/* NormRow, CachedRowMath.ts:25-56 (LayerNormRow / RmsNormRow). */
static void NormRow(const OracleModel* m, const double* g, const double* b, const double* x, double* out) {
  const int N = m->E;
  const double eps = m->cfg.layer_norm_eps;
  if (m->cfg.norm_kind == 1) {
    double ss = 0;
    for (int j = 0; j < N; j++) ss += x[j] * x[j];
    double is = 1.0 / sqrt(ss / N + eps);
    for (int j = 0; j < N; j++) out[j] = g[j] * x[j] * is;
    return;
  }
  double mu = 0;
  for (int j = 0; j < N; j++) mu += x[j];
  mu /= N;
  double var = 0;
  for (int j = 0; j < N; j++) {
    double dd = x[j] - mu;
    var += dd * dd;
  }
  var /= N;
  double is = 1.0 / sqrt(var + eps);
  for (int j = 0; j < N; j++) out[j] = g[j] * ((x[j] - mu) * is) + b[j];
}

/* RotateRow, RotaryEmbedding.ts:42-60 (interleaved pairs (2i, 2i+1)). */
static void RotateRow(double* row, const double* cs, const double* sn, int half) {
  for (int i = 0; i < half; i++) {
    double c = cs[i], s = sn[i];
    double x0 = row[2 * i], x1 = row[2 * i + 1];
    row[2 * i] = x0 * c - x1 * s;
    row[2 * i + 1] = x0 * s + x1 * c;
  }
}

/* AttendRow, CachedRowMath.ts:60-86. */
static void AttendRow(const double* q, const double* keys, const double* values, int T, int d, double scale,
                      double* scores, double* ctx) {
  double mx = -INFINITY;
  for (int t = 0; t < T; t++) {
    double dot = 0;
    for (int j = 0; j < d; j++) dot += q[j] * keys[(size_t)t * d + j];
    double sc = dot * scale;
    scores[t] = sc;
    if (sc > mx) mx = sc;
  }
  double sum = 0;
  for (int t = 0; t < T; t++) {
    double ex = exp(scores[t] - mx);
    scores[t] = ex;
    sum += ex;
  }
  for (int j = 0; j < d; j++) ctx[j] = 0;
  for (int t = 0; t < T; t++) {
    double w = scores[t] / sum;
    if (w == 0) continue;
    for (int j = 0; j < d; j++) ctx[j] += w * values[(size_t)t * d + j];
  }
}

/* SiluValue (Silu.ts:8-10) and GeluValue (Gelu.ts:7-14). */
static double SiluValue(double v) { return v * (1.0 / (1.0 + exp(-v))); }
static double GeluValue(double v) {
  const double c = sqrt(2.0 / M_PI);
  double inner = c * (v + 0.044715 * v * v * v);
  return 0.5 * v * (1.0 + tanh(inner));
}

/* MlpRow, CachedRowMath.ts:94-114. */
static void MlpRow(const OracleModel* m, const LayerOff* L, const double* x, double* out, double* h1, double* h2) {
  const int E = m->E, F = m->F;
  const double* p = m->p;
  if (m->cfg.mlp_kind == 0) {
    MatMulRow(x, p + L->wfc, E, F, h1);
    for (int j = 0; j < F; j++) {
      double v = h1[j] + p[L->bfc + j];
      h1[j] = v > 0 ? v : 0;
    }
    MatMulRow(h1, p + L->wproj, F, E, out);
    for (int j = 0; j < E; j++) out[j] += p[L->bproj + j];
    return;
  }
  MatMulRow(x, p + L->w1, E, F, h1);
  MatMulRow(x, p + L->w3, E, F, h2);
  for (int j = 0; j < F; j++) h1[j] = (m->cfg.mlp_kind == 1 ? SiluValue(h1[j]) : GeluValue(h1[j])) * h2[j];
  MatMulRow(h1, p + L->w2, F, E, out);
}

/* HeadLogitsRow, CachedRowMath.ts:117-137. */
static void HeadLogitsRow(const OracleModel* m, const double* x, double* logits, double* xf) {
  const int E = m->E, V = m->V;
  const double* p = m->p;
  NormRow(m, p + m->lay.lnf_g, m->lay.lnf_b >= 0 ? p + m->lay.lnf_b : NULL, x, xf);
  const double* bias = p + m->lay.lm_bias;
  if (!m->cfg.weight_tying) {
    MatMulRow(xf, p + m->lay.lm_head, E, V, logits);
    for (int v = 0; v < V; v++) logits[v] += bias[v];
    return;
  }
  const double* wte = p + m->lay.wte;
  for (int v = 0; v < V; v++) {
    double s = 0;
    for (int j = 0; j < E; j++) s += xf[j] * wte[(size_t)v * E + j];
    logits[v] = s + bias[v];
  }
}

/* AdvanceOneToken + CachedForwardStep, CachedForward.ts:32-96. */
int oracle_cached_step(const OracleModel* m, OracleCache* c, int token, int position, double* logits) {
  const int E = m->E, d = m->d, F = m->F;
  if (token < 0 || token >= m->V)
    return Fail("CachedForwardStep: token id %d out of range [0,%d)", token, m->V);
  if (position != oracle_cache_length(c))
    return Fail("CachedForwardStep: position %d must equal the cached length %d (positions are contiguous)", position,
                oracle_cache_length(c));
  if (position >= c->C) return Fail("CachedForwardStep: position %d is outside the %d-token window", position, c->C);
  if (m->lay.wpe >= 0 && position >= m->C) return Fail("CachedForwardStep: position %d has no learned embedding", position);
  const double* p = m->p;
  double* x = (double*)malloc(sizeof(double) * E);
  double* xn = (double*)malloc(sizeof(double) * E);
  double* attn = (double*)malloc(sizeof(double) * E);
  double* proj = (double*)malloc(sizeof(double) * E);
  double* k = (double*)malloc(sizeof(double) * d);
  double* v = (double*)malloc(sizeof(double) * d);
  double* q = (double*)malloc(sizeof(double) * d);
  double* ctx = (double*)malloc(sizeof(double) * d);
  double* scores = (double*)malloc(sizeof(double) * (size_t)c->C);
  double* h1 = (double*)malloc(sizeof(double) * F);
  double* h2 = (double*)malloc(sizeof(double) * F);
  double* cs = (double*)malloc(sizeof(double) * (d / 2 + 1));
  double* sn = (double*)malloc(sizeof(double) * (d / 2 + 1));
  for (int j = 0; j < E; j++) x[j] = p[m->lay.wte + (int64_t)token * E + j];
  if (m->lay.wpe >= 0)
    for (int j = 0; j < E; j++) x[j] += p[m->lay.wpe + (int64_t)position * E + j];
  const int rope = m->cfg.position_scheme == 1;
  if (rope) /* RopeCosSin, RotaryEmbedding.ts:25-38 */
    for (int i = 0; i < d / 2; i++) {
      double ang = position * m->freq[i];
      cs[i] = cos(ang);
      sn[i] = sin(ang);
    }
  int rc = 0;
  for (int l = 0; l < m->L && rc == 0; l++) {
    const LayerOff* L = &m->lay.layers[l];
    NormRow(m, p + L->ln1_g, L->ln1_b >= 0 ? p + L->ln1_b : NULL, x, xn);
    for (int g = 0; g < m->Hk; g++) {
      MatMulRow(xn, p + L->wk + (int64_t)g * E * d, E, d, k);
      if (rope) RotateRow(k, cs, sn, d / 2);
      MatMulRow(xn, p + L->wv + (int64_t)g * E * d, E, d, v);
      rc = CacheAppendRows(c, l, g, k, v, 1);
      if (rc) break;
    }
    if (rc) break;
    for (int j = 0; j < E; j++) attn[j] = 0;
    for (int h = 0; h < m->H; h++) {
      int kv = h / m->G;
      MatMulRow(xn, p + L->wq + (int64_t)h * E * d, E, d, q);
      if (rope) RotateRow(q, cs, sn, d / 2);
      int idx = l * m->Hk + kv;
      size_t base = (size_t)idx * c->C * d;
      AttendRow(q, c->keys + base, c->values + base, c->lengths[idx], d, m->scale, scores, ctx);
      MatMulRow(ctx, p + L->wo + (int64_t)h * d * E, d, E, proj);
      for (int j = 0; j < E; j++) attn[j] += proj[j];
    }
    for (int j = 0; j < E; j++) x[j] += attn[j];
    NormRow(m, p + L->ln2_g, L->ln2_b >= 0 ? p + L->ln2_b : NULL, x, xn);
    MlpRow(m, L, xn, proj, h1, h2);
    for (int j = 0; j < E; j++) x[j] += proj[j];
  }
  if (rc == 0) HeadLogitsRow(m, x, logits, xn);
  free(x); free(xn); free(attn); free(proj); free(k); free(v); free(q); free(ctx); free(scores);
  free(h1); free(h2); free(cs); free(sn);
  return rc;
}

/* ------------------------------------------------------------------------------------------------
 * Tensor forward (Shahd.ForwardHidden / Forward): ops of Brain/Ops with the run's storage rounding.
 * ---------------------------------------------------------------------------------------------- */

#define ST(x) (f32 ? StoreF32(x) : (x))

/* Intra-op threads of the tensor matmul (1 = serial). Rows are split across threads and handled in
 * blocks of 4 that share each streamed row of B; every output element still accumulates over pp in
 * ascending order, so results do not depend on the thread count. */
static int g_oracle_threads = 1;
void oracle_set_threads(int n) { g_oracle_threads = n < 1 ? 1 : n; }

typedef struct TMatJob {
  const double *a, *b;
  double* out;
  int i0, i1, K, N, f32;
} TMatJob;

/* MatMul inline path, Ops/MatMul.ts:60-73: Out += AVal * B with the zero skip; each += stores. */
static void TMatMulRows(const double* a, const double* b, double* out, int i0, int i1, int K, int N, int f32) {
  memset(out + (size_t)i0 * N, 0, sizeof(double) * (size_t)(i1 - i0) * N);
  for (int ib = i0; ib < i1; ib += 4) {
    const int ie = ib + 4 < i1 ? ib + 4 : i1;
    for (int pp = 0; pp < K; pp++) {
      const double* br = b + (size_t)pp * N;
      for (int i = ib; i < ie; i++) {
        double av = a[(size_t)i * K + pp];
        if (av == 0) continue;
        double* o = out + (size_t)i * N;
        if (f32)
          for (int j = 0; j < N; j++) o[j] = StoreF32(o[j] + av * br[j]);
        else
          for (int j = 0; j < N; j++) o[j] = o[j] + av * br[j];
      }
    }
  }
}

static void* TMatWorker(void* arg) {
  TMatJob* j = (TMatJob*)arg;
  TMatMulRows(j->a, j->b, j->out, j->i0, j->i1, j->K, j->N, j->f32);
  return NULL;
}

static void TMatMul(const double* a, const double* b, double* out, int M, int K, int N, int f32) {
  int nt = g_oracle_threads;
  if (nt > M / 4) nt = M / 4;
  if (nt <= 1 || (double)M * K * N < 4e6) {
    TMatMulRows(a, b, out, 0, M, K, N, f32);
    return;
  }
  pthread_t th[64];
  TMatJob jobs[64];
  if (nt > 64) nt = 64;
  const int per = ((M + nt - 1) / nt + 3) / 4 * 4;
  int n = 0;
  for (int i0 = 0; i0 < M; i0 += per, n++) {
    jobs[n] = (TMatJob){a, b, out, i0, i0 + per < M ? i0 + per : M, K, N, f32};
    pthread_create(&th[n], NULL, TMatWorker, &jobs[n]);
  }
  for (int t = 0; t < n; t++) pthread_join(th[t], NULL);
}

/* MatMulNT InlineForward, Ops/MatMulNT.ts:27-43: p-ascending dot from zero, one store. */
static void TMatMulNT(const double* a, const double* bt, double* out, int M, int K, int N, int f32) {
  for (int i = 0; i < M; i++)
    for (int j = 0; j < N; j++) {
      double s = 0;
      for (int pp = 0; pp < K; pp++) s += a[(size_t)i * K + pp] * bt[(size_t)j * K + pp];
      out[(size_t)i * N + j] = ST(s);
    }
}

/* NormLayer.Forward (NormLayer.ts:22-26) over rows: RmsNorm.ts:19-29 / LayerNorm.ts:23-41. */
static void TNorm(const OracleModel* m, const double* g, const double* b, const double* x, double* out, int T) {
  const int N = m->E, f32 = m->cfg.precision_f32;
  const double eps = m->cfg.layer_norm_eps;
  for (int i = 0; i < T; i++) {
    const double* xr = x + (size_t)i * N;
    double* o = out + (size_t)i * N;
    if (m->cfg.norm_kind == 1) {
      double ss = 0;
      for (int j = 0; j < N; j++) ss += xr[j] * xr[j];
      double is = 1.0 / sqrt(ss / N + eps);
      for (int j = 0; j < N; j++) o[j] = ST(g[j] * xr[j] * is);
    } else {
      double mu = 0;
      for (int j = 0; j < N; j++) mu += xr[j];
      mu /= N;
      double var = 0;
      for (int j = 0; j < N; j++) {
        double dd = xr[j] - mu;
        var += dd * dd;
      }
      var /= N;
      double is = 1.0 / sqrt(var + eps);
      for (int j = 0; j < N; j++) o[j] = ST(g[j] * ((xr[j] - mu) * is) + b[j]);
    }
  }
}

/* ApplyRope(X, 0), RotaryEmbedding.ts:63-75. */
static void TRope(const OracleModel* m, double* x, int T) {
  const int d = m->d, half = d / 2, f32 = m->cfg.precision_f32;
  for (int r = 0; r < T; r++) {
    double* row = x + (size_t)r * d;
    for (int i = 0; i < half; i++) {
      double ang = r * m->freq[i];
      double c = cos(ang), s = sin(ang);
      double x0 = row[2 * i], x1 = row[2 * i + 1];
      row[2 * i] = ST(x0 * c - x1 * s);
      row[2 * i + 1] = ST(x0 * s + x1 * c);
    }
  }
}

/* CausalSoftmax, CausalSoftmax.ts:17-33, with ComputeRowSoftmax (Internal/RowSoftmax.ts:14-31). */
static void TCausalSoftmax(double* s, int T, double factor, int f32) {
  for (int i = 0; i < T; i++) {
    double* row = s + (size_t)i * T;
    int vis = i + 1;
    for (int j = 0; j < vis; j++) row[j] = ST(row[j] * factor);
    double mx = -INFINITY;
    for (int j = 0; j < vis; j++) mx = fmax(mx, row[j]);
    double sum = 0;
    for (int j = 0; j < vis; j++) {
      double e = exp(row[j] - mx);
      row[j] = ST(e);
      sum += e;
    }
    for (int j = 0; j < vis; j++) row[j] = ST(row[j] / sum);
    for (int j = vis; j < T; j++) row[j] = 0;
  }
}

/* Shahd.ForwardHidden (Shahd.ts:43-55) with an optional KV sink into a cache (PrefillCache). */
static int ForwardHidden(const OracleModel* m, const int32_t* ids, int T, double* x, OracleCache* sink) {
  const int E = m->E, d = m->d, F = m->F, f32 = m->cfg.precision_f32;
  const double* p = m->p;
  if (T > m->C) return Fail("Shahd.Forward: sequence length %d exceeds BlockSize %d", T, m->C);
  for (int i = 0; i < T; i++)
    if (ids[i] < 0 || ids[i] >= m->V) return Fail("EmbeddingLookup: id %d at position %d out of range [0,%d)", ids[i], i, m->V);
  /* Embedding.Forward, Embedding.ts:20-26 */
  for (int i = 0; i < T; i++)
    for (int j = 0; j < E; j++) {
      double t = p[m->lay.wte + (int64_t)ids[i] * E + j];
      x[(size_t)i * E + j] = m->lay.wpe >= 0 ? ST(t + p[m->lay.wpe + (int64_t)i * E + j]) : t;
    }
  size_t TE = (size_t)T * E, Td = (size_t)T * d, TF = (size_t)T * F;
  double* xn = (double*)malloc(sizeof(double) * TE);
  double* out = (double*)malloc(sizeof(double) * TE);
  double* proj = (double*)malloc(sizeof(double) * TE);
  double* ks = (double*)malloc(sizeof(double) * Td * m->Hk);
  double* vs = (double*)malloc(sizeof(double) * Td * m->Hk);
  double* q = (double*)malloc(sizeof(double) * Td);
  double* sc = (double*)malloc(sizeof(double) * (size_t)T * T);
  double* ho = (double*)malloc(sizeof(double) * Td);
  double* h1 = (double*)malloc(sizeof(double) * TF);
  double* h2 = (double*)malloc(sizeof(double) * TF);
  int rc = 0;
  for (int l = 0; l < m->L && rc == 0; l++) {
    const LayerOff* L = &m->lay.layers[l];
    /* Block.Forward, Block.ts:28-32; MultiHeadAttention.Forward, MultiHeadAttention.ts:46-74 */
    TNorm(m, p + L->ln1_g, L->ln1_b >= 0 ? p + L->ln1_b : NULL, x, xn, T);
    for (int g = 0; g < m->Hk; g++) {
      double* K = ks + Td * g;
      double* V = vs + Td * g;
      TMatMul(xn, p + L->wk + (int64_t)g * E * d, K, T, E, d, f32);
      if (m->cfg.position_scheme == 1) TRope(m, K, T);
      TMatMul(xn, p + L->wv + (int64_t)g * E * d, V, T, E, d, f32);
      if (sink) {
        rc = CacheAppendRows(sink, l, g, K, V, T);
        if (rc) break;
      }
    }
    if (rc) break;
    for (int h = 0; h < m->H; h++) {
      int kv = h / m->G;
      TMatMul(xn, p + L->wq + (int64_t)h * E * d, q, T, E, d, f32);
      if (m->cfg.position_scheme == 1) TRope(m, q, T);
      TMatMulNT(q, ks + Td * kv, sc, T, d, T, f32);
      TCausalSoftmax(sc, T, m->scale, f32);
      TMatMul(sc, vs + Td * kv, ho, T, T, d, f32);
      TMatMul(ho, p + L->wo + (int64_t)h * d * E, proj, T, d, E, f32);
      if (h == 0) memcpy(out, proj, sizeof(double) * TE);
      else
        for (size_t i = 0; i < TE; i++) out[i] = ST(out[i] + proj[i]);
    }
    for (size_t i = 0; i < TE; i++) x[i] = ST(x[i] + out[i]);
    /* Mlp.Forward, Mlp.ts:43-57 */
    TNorm(m, p + L->ln2_g, L->ln2_b >= 0 ? p + L->ln2_b : NULL, x, xn, T);
    if (m->cfg.mlp_kind == 0) {
      TMatMul(xn, p + L->wfc, h1, T, E, F, f32);
      for (size_t i = 0; i < TF; i++) {
        double v = ST(h1[i] + p[L->bfc + (int64_t)(i % F)]);
        h1[i] = v > 0 ? v : 0;
      }
      TMatMul(h1, p + L->wproj, out, T, F, E, f32);
      for (size_t i = 0; i < TE; i++) out[i] = ST(out[i] + p[L->bproj + (int64_t)(i % E)]);
    } else {
      TMatMul(xn, p + L->w1, h1, T, E, F, f32);
      for (size_t i = 0; i < TF; i++) h1[i] = ST(m->cfg.mlp_kind == 1 ? SiluValue(h1[i]) : GeluValue(h1[i]));
      TMatMul(xn, p + L->w3, h2, T, E, F, f32);
      for (size_t i = 0; i < TF; i++) h1[i] = ST(h1[i] * h2[i]);
      TMatMul(h1, p + L->w2, out, T, F, E, f32);
    }
    for (size_t i = 0; i < TE; i++) x[i] = ST(x[i] + out[i]);
  }
  free(xn); free(out); free(proj); free(ks); free(vs); free(q); free(sc); free(ho); free(h1); free(h2);
  return rc;
}

/* Shahd.Head (Shahd.ts:77-84) on normalized rows. */
static void THead(const OracleModel* m, const double* xf, int T, double* logits) {
  const int f32 = m->cfg.precision_f32, V = m->V, E = m->E;
  const double* p = m->p;
  if (m->cfg.weight_tying) TMatMulNT(xf, p + m->lay.wte, logits, T, E, V, f32);
  else TMatMul(xf, p + m->lay.lm_head, logits, T, E, V, f32);
  for (int i = 0; i < T; i++)
    for (int v = 0; v < V; v++) logits[(size_t)i * V + v] = ST(logits[(size_t)i * V + v] + p[m->lay.lm_bias + v]);
}

int oracle_forward(const OracleModel* m, const int32_t* ids, int T, double* logits) {
  if (T <= 0) return Fail("Shahd.Forward: empty input");
  double* x = (double*)malloc(sizeof(double) * (size_t)T * m->E);
  double* xf = (double*)malloc(sizeof(double) * (size_t)T * m->E);
  int rc = ForwardHidden(m, ids, T, x, NULL);
  if (rc == 0) {
    TNorm(m, m->p + m->lay.lnf_g, m->lay.lnf_b >= 0 ? m->p + m->lay.lnf_b : NULL, x, xf, T);
    THead(m, xf, T, logits);
  }
  free(x); free(xf);
  return rc;
}

int oracle_forward_last_logits(const OracleModel* m, const int32_t* ids, int T, double* logits) {
  if (T <= 0) return Fail("Shahd.ForwardLastLogits: empty context — nothing to predict from");
  double* x = (double*)malloc(sizeof(double) * (size_t)T * m->E);
  double* xf = (double*)malloc(sizeof(double) * (size_t)m->E);
  int rc = ForwardHidden(m, ids, T, x, NULL);
  if (rc == 0) {
    TNorm(m, m->p + m->lay.lnf_g, m->lay.lnf_b >= 0 ? m->p + m->lay.lnf_b : NULL, x + (size_t)(T - 1) * m->E, xf, 1);
    THead(m, xf, 1, logits);
  }
  free(x); free(xf);
  return rc;
}

/* PrefillCache, CachedForward.ts:100-110. */
int oracle_prefill(const OracleModel* m, OracleCache* c, const int32_t* ids, int n) {
  CacheReset(c);
  if (n == 0) return 0;
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= m->V) return Fail("PrefillCache: token id %d out of range [0,%d)", ids[i], m->V);
  if (n > c->C) return Fail("PrefillCache: %d tokens exceed the cache capacity %d", n, c->C);
  double* x = (double*)malloc(sizeof(double) * (size_t)n * m->E);
  int rc = ForwardHidden(m, ids, n, x, c);
  free(x);
  return rc;
}

/* ------------------------------------------------------------------------------------------------
 * Sampling: Brain/Sampling/Distribution.ts, Sampler.ts
 * ---------------------------------------------------------------------------------------------- */

/* ArgmaxOf, Distribution.ts:19-30: first index of the strict max. */
int oracle_argmax(const double* logits, int V) {
  int best = 0;
  double bv = -INFINITY;
  for (int j = 0; j < V; j++)
    if (logits[j] > bv) {
      bv = logits[j];
      best = j;
    }
  return best;
}

typedef struct SortKey {
  double p;
  int idx;
} SortKey;

/* Array.prototype.sort with (A, B) => Probs[B] - Probs[A] is stable: descending probability, ties in
 * ascending index order. */
static int CmpDesc(const void* a, const void* b) {
  const SortKey* x = (const SortKey*)a;
  const SortKey* y = (const SortKey*)b;
  if (x->p > y->p) return -1;
  if (x->p < y->p) return 1;
  return x->idx < y->idx ? -1 : (x->idx > y->idx);
}

/* ProbsFromLogits, Distribution.ts:35-89. */
void oracle_probs_from_logits(const double* logits, int V, const OracleSampling* o, double* probs) {
  if (o->temperature <= 0) {
    for (int j = 0; j < V; j++) probs[j] = 0;
    probs[oracle_argmax(logits, V)] = 1;
    return;
  }
  double mx = -INFINITY;
  for (int j = 0; j < V; j++) {
    double s = logits[j] / o->temperature;
    probs[j] = s;
    if (s > mx) mx = s;
  }
  double sum = 0;
  for (int j = 0; j < V; j++) {
    double e = exp(probs[j] - mx);
    probs[j] = e;
    sum += e;
  }
  for (int j = 0; j < V; j++) probs[j] /= sum;
  if (o->top_k <= 0 && o->top_p >= 1) return;
  SortKey* keys = (SortKey*)malloc(sizeof(SortKey) * (size_t)V);
  for (int j = 0; j < V; j++) {
    keys[j].p = probs[j];
    keys[j].idx = j;
  }
  qsort(keys, (size_t)V, sizeof(SortKey), CmpDesc);
  int kept = V;
  if (o->top_k > 0 && o->top_k < kept) kept = o->top_k;
  if (o->top_p < 1) {
    double mass = 0;
    for (int i = 0; i < kept; i++) mass += keys[i].p;
    double thr = o->top_p * mass;
    double cum = 0;
    int n = 0;
    for (int i = 0; i < kept; i++) {
      n++;
      cum += keys[i].p;
      if (cum >= thr) break;
    }
    kept = n;
  }
  double ks = 0;
  for (int i = 0; i < kept; i++) ks += keys[i].p;
  double* outp = (double*)calloc((size_t)V, sizeof(double));
  if (ks > 0)
    for (int i = 0; i < kept; i++) outp[keys[i].idx] = keys[i].p / ks;
  memcpy(probs, outp, sizeof(double) * (size_t)V);
  free(outp);
  free(keys);
}

/* SampleFromDistribution, Distribution.ts:93-104. */
int oracle_sample_from_distribution(const double* probs, int V, uint32_t* rng) {
  int last = -1;
  double r = oracle_rng_next_float(rng);
  for (int j = 0; j < V; j++) {
    double pj = probs[j];
    if (pj <= 0) continue;
    last = j;
    r -= pj;
    if (r <= 0) return j;
  }
  return last >= 0 ? last : 0;
}

/* SampleFromLogits, Sampler.ts:16-27. */
int oracle_sample_from_logits(const double* logits, int V, const OracleSampling* o, uint32_t* rng) {
  if (o->temperature <= 0) return oracle_argmax(logits, V);
  double* probs = (double*)malloc(sizeof(double) * (size_t)V);
  oracle_probs_from_logits(logits, V, o, probs);
  int id = oracle_sample_from_distribution(probs, V, rng);
  free(probs);
  return id;
}

/* ------------------------------------------------------------------------------------------------
 * CachedDecoder (CachedForward.ts:113-150) and the generation loops
 * ---------------------------------------------------------------------------------------------- */

struct OracleDecoder {
  const OracleModel* m;
  OracleCache* cache;
  int32_t* window; /* ids currently in the cache, oldest first */
  int wlen;
  double* logits;
};

static int DecoderStep(OracleDecoder* d, int token) {
  int rc = oracle_cached_step(d->m, d->cache, token, oracle_cache_length(d->cache), d->logits);
  if (rc == 0) d->window[d->wlen++] = token;
  return rc;
}

OracleDecoder* oracle_decoder_create(const OracleModel* m, const int32_t* prompt, int n) {
  if (n <= 0) {
    Fail("CachedDecoder: empty prompt — nothing to condition on");
    return NULL;
  }
  OracleDecoder* d = (OracleDecoder*)calloc(1, sizeof(OracleDecoder));
  d->m = m;
  d->cache = oracle_cache_create(m);
  d->window = (int32_t*)malloc(sizeof(int32_t) * (size_t)(m->C + 1));
  d->logits = (double*)malloc(sizeof(double) * (size_t)m->V);
  int ctx = n < m->C ? n : m->C;
  const int32_t* context = prompt + (n - ctx); /* PromptIds.slice(-BlockSize) */
  int rc = oracle_prefill(m, d->cache, context, ctx - 1);
  if (rc == 0) {
    memcpy(d->window, context, sizeof(int32_t) * (size_t)(ctx - 1));
    d->wlen = ctx - 1;
    rc = DecoderStep(d, context[ctx - 1]);
  }
  if (rc) {
    oracle_decoder_destroy(d);
    return NULL;
  }
  return d;
}

int oracle_decoder_push(OracleDecoder* d, int token) {
  if (token < 0 || token >= d->m->V) return Fail("CachedDecoder.Push: token id %d out of range [0,%d)", token, d->m->V);
  if (oracle_cache_length(d->cache) >= d->cache->C) {
    int keep = d->cache->C - 1; /* Window.slice(-(Capacity - 1)) */
    if (keep > d->wlen) keep = d->wlen;
    int32_t* tmp = (int32_t*)malloc(sizeof(int32_t) * (size_t)(keep + 1));
    memcpy(tmp, d->window + (d->wlen - keep), sizeof(int32_t) * (size_t)keep);
    int rc = oracle_prefill(d->m, d->cache, tmp, keep);
    memcpy(d->window, tmp, sizeof(int32_t) * (size_t)keep);
    d->wlen = keep;
    free(tmp);
    if (rc) return rc;
  }
  return DecoderStep(d, token);
}

const double* oracle_decoder_logits(const OracleDecoder* d) { return d->logits; }
int oracle_decoder_cache_length(const OracleDecoder* d) { return oracle_cache_length(d->cache); }

void oracle_decoder_destroy(OracleDecoder* d) {
  if (!d) return;
  oracle_cache_destroy(d->cache);
  free(d->window);
  free(d->logits);
  free(d);
}

/* CachedGenerate, CachedForward.ts:153-171. */
int oracle_cached_generate(const OracleModel* m, const int32_t* prompt, int n, int max_new, const OracleSampling* o,
                           uint32_t* rng, int32_t* out) {
  if (n <= 0) return Fail("CachedGenerate: empty prompt — nothing to condition on");
  memcpy(out, prompt, sizeof(int32_t) * (size_t)n);
  if (!(max_new >= 1)) return 0;
  OracleDecoder* d = oracle_decoder_create(m, prompt, n);
  if (!d) return -1;
  int rc = 0;
  for (int s = 0; s < max_new; s++) {
    int next = oracle_sample_from_logits(d->logits, m->V, o, rng);
    out[n + s] = next;
    if (s + 1 < max_new) {
      rc = oracle_decoder_push(d, next);
      if (rc) break;
    }
  }
  oracle_decoder_destroy(d);
  return rc;
}

/* Generate + StepToken, Generate.ts:17-43. */
int oracle_generate(const OracleModel* m, const int32_t* prompt, int n, int max_new, const OracleSampling* o,
                    uint32_t* rng, int32_t* out) {
  if (n <= 0) return Fail("Generate: empty prompt — nothing to condition on");
  memcpy(out, prompt, sizeof(int32_t) * (size_t)n);
  double* logits = (double*)malloc(sizeof(double) * (size_t)m->V);
  int len = n, rc = 0;
  for (int s = 0; s < max_new; s++) {
    int t = len < m->C ? len : m->C;
    rc = oracle_forward_last_logits(m, out + (len - t), t, logits);
    if (rc) break;
    out[len++] = oracle_sample_from_logits(logits, m->V, o, rng);
  }
  free(logits);
  return rc;
}

typedef struct BatchJob {
  const OracleModel* m;
  const int32_t* prompts;
  int nseq, plen, max_new, threads, tid, rc;
  const OracleSampling* o;
  uint32_t* rng;
  int32_t* out;
} BatchJob;

static void* BatchWorker(void* arg) {
  BatchJob* j = (BatchJob*)arg;
  for (int s = j->tid; s < j->nseq; s += j->threads) {
    int rc = oracle_cached_generate(j->m, j->prompts + (size_t)s * j->plen, j->plen, j->max_new, j->o, &j->rng[s],
                                    j->out + (size_t)s * (j->plen + j->max_new));
    if (rc) j->rc = rc;
  }
  return NULL;
}

int oracle_cached_generate_batch(const OracleModel* m, const int32_t* prompts, int nseq, int plen, int max_new,
                                 const OracleSampling* o, uint32_t* rng, int32_t* out, int threads) {
  if (threads < 1) threads = 1;
  if (threads > nseq) threads = nseq;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  BatchJob* jobs = (BatchJob*)malloc(sizeof(BatchJob) * (size_t)threads);
  for (int t = 0; t < threads; t++) {
    jobs[t] = (BatchJob){m, prompts, nseq, plen, max_new, threads, t, 0, o, rng, out};
    pthread_create(&th[t], NULL, BatchWorker, &jobs[t]);
  }
  int rc = 0;
  for (int t = 0; t < threads; t++) {
    pthread_join(th[t], NULL);
    if (jobs[t].rc) rc = jobs[t].rc;
  }
  free(th);
  free(jobs);
  return rc;
}

/* ---- teacher-forced check of externally produced greedy trajectories ----------------------------
 * For sequence s a CachedDecoder (CachedForward.ts:113-150) is built from prompts[s]; at step k the
 * oracle's logits, given prompt ++ ids[s][0..k), judge ids[s][k]: it passes when it is the oracle's
 * ArgmaxOf (Distribution.ts:19-30), or when the oracle's top-2 margin is within tol x (max - min), a near
 * tie where a rounding difference may pick either id. ids[s][k] is then pushed, so every step is judged
 * on the checked implementation's own prefix. Outputs per sequence: failing steps, the first failing
 * step (-1: none), near ties met with a different id, and the largest gap (max logit - logit of the
 * chosen id) relative to the logit range. */
typedef struct CheckJob {
  const OracleModel* m;
  const int32_t* prompts;
  const int32_t* ids;
  int nseq, plen, nnew, threads, tid, rc;
  double tol;
  int32_t *fails, *first_fail, *near_ties;
  double* max_gap;
} CheckJob;

static void* CheckWorker(void* arg) {
  CheckJob* j = (CheckJob*)arg;
  const int V = j->m->V;
  for (int s = j->tid; s < j->nseq; s += j->threads) {
    const int32_t* ids = j->ids + (size_t)s * j->nnew;
    int fails = 0, first = -1, ties = 0;
    double worst = 0.0;
    OracleDecoder* d = oracle_decoder_create(j->m, j->prompts + (size_t)s * j->plen, j->plen);
    if (!d) {
      j->rc = -1;
      continue;
    }
    for (int k = 0; k < j->nnew; k++) {
      const double* lg = d->logits;
      const int tok = ids[k];
      if (tok < 0 || tok >= V) {
        fails++;
        if (first < 0) first = k;
        break;
      }
      double mx = -INFINITY, mn = INFINITY, second = -INFINITY;
      int am = oracle_argmax(lg, V);
      for (int v = 0; v < V; v++) {
        if (lg[v] > mx) mx = lg[v];
        if (lg[v] < mn) mn = lg[v];
        if (v != am && lg[v] > second) second = lg[v];
      }
      const double range = mx - mn > 0 ? mx - mn : 1e-300;
      const double gap = (mx - lg[tok]) / range;
      if (gap > worst) worst = gap;
      if (tok != am) {
        if (mx - second <= j->tol * range && gap <= j->tol) {
          ties++;
        } else {
          fails++;
          if (first < 0) first = k;
        }
      }
      if (k + 1 < j->nnew && oracle_decoder_push(d, tok) != 0) {
        j->rc = -1;
        break;
      }
    }
    oracle_decoder_destroy(d);
    j->fails[s] = fails;
    j->first_fail[s] = first;
    j->near_ties[s] = ties;
    j->max_gap[s] = worst;
  }
  return NULL;
}

int oracle_check_trajectories(const OracleModel* m, const int32_t* prompts, int nseq, int plen, const int32_t* ids,
                              int nnew, double tol, int threads, int32_t* fails, int32_t* first_fail,
                              int32_t* near_ties, double* max_gap) {
  if (threads < 1) threads = 1;
  if (threads > nseq) threads = nseq;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  CheckJob* jobs = (CheckJob*)malloc(sizeof(CheckJob) * (size_t)threads);
  for (int t = 0; t < threads; t++) {
    jobs[t] = (CheckJob){m, prompts, ids, nseq, plen, nnew, threads, t, 0, tol, fails, first_fail, near_ties, max_gap};
    pthread_create(&th[t], NULL, CheckWorker, &jobs[t]);
  }
  int rc = 0;
  for (int t = 0; t < threads; t++) {
    pthread_join(th[t], NULL);
    if (jobs[t].rc) rc = jobs[t].rc;
  }
  free(th);
  free(jobs);
  return rc;
}

/* ---- stochastic speculative sampling (Brain/Reasoning/SpeculativeSampling.ts) ------------------- */

/* ResidualSample, SpeculativeSampling.ts:23-36: a draw from the normalized max(0, P - Q), or from P when
 * that residual has no mass. */
static int ResidualSample(const double* P, const double* Q, int V, uint32_t* rng, double* tmp) {
  double sum = 0;
  for (int j = 0; j < V; j++) {
    const double r = P[j] - Q[j];
    tmp[j] = r > 0 ? r : 0;
    if (r > 0) sum += r;
  }
  if (sum <= 0) return oracle_sample_from_distribution(P, V, rng);
  for (int j = 0; j < V; j++) tmp[j] /= sum;
  return oracle_sample_from_distribution(tmp, V, rng);
}

/* One verification round (SpeculativeSampling.ts:82-112) on given logits: target rows [g + 1][V] (row i is
 * the target's prediction for proposal i, row g the bonus position), draft rows [g][V] (row i is the
 * distribution proposal i was drawn from). Appends the round's ids to out (at most budget of them) and
 * returns their count; *accepted receives the accepted proposals. One Rng draw per examined proposal, one
 * more for the residual or bonus sample, in the reference's order. */
int oracle_speculative_round(const double* target, const double* draft, const int32_t* proposals, int g, int V,
                             int budget, const OracleSampling* o, uint32_t* rng, int32_t* out, int* accepted) {
  double* P = (double*)malloc(sizeof(double) * (size_t)V);
  double* Q = (double*)malloc(sizeof(double) * (size_t)V);
  double* T = (double*)malloc(sizeof(double) * (size_t)V);
  int n = 0, acc = 0, corrected = 0;
  for (int i = 0; i < g; i++) {
    oracle_probs_from_logits(target + (size_t)i * V, V, o, P);
    oracle_probs_from_logits(draft + (size_t)i * V, V, o, Q);
    const int tok = proposals[i];
    const double ratio = Q[tok] > 0 ? P[tok] / Q[tok] : (P[tok] > 0 ? 1 : 0);
    if (oracle_rng_next_float(rng) < (ratio < 1 ? ratio : 1)) {
      out[n++] = tok;
      acc++;
      if (n >= budget) break;
    } else {
      out[n++] = ResidualSample(P, Q, V, rng, T);
      corrected = 1;
      break;
    }
  }
  if (!corrected && n < budget) {
    oracle_probs_from_logits(target + (size_t)g * V, V, o, P);
    out[n++] = oracle_sample_from_distribution(P, V, rng);
  }
  free(P);
  free(Q);
  free(T);
  *accepted = acc;
  return n;
}

/* SpeculativeSample, SpeculativeSampling.ts:38-115: the draft proposes from ForwardLastLogits of its window,
 * the target scores [ids, proposals].slice(-BlockSize) in one Forward. out_ids receives prompt + max_new ids;
 * stats (nullable) [target calls, draft tokens, accepted tokens]. */
int oracle_speculative_sample(const OracleModel* target, const OracleModel* draft, const int32_t* prompt, int n,
                              int max_new, const OracleSampling* o, uint32_t* rng, int gamma, int32_t* out_ids,
                              int32_t* stats) {
  if (n <= 0) return Fail("SpeculativeSample: empty prompt");
  const int V = target->V, C = target->C, DC = draft->C;
  int32_t* ids = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + max_new + gamma + 2));
  memcpy(ids, prompt, sizeof(int32_t) * (size_t)n);
  int len = n, calls = 0, dtok = 0, acc_total = 0, rc = 0;
  double* dl = (double*)malloc(sizeof(double) * (size_t)gamma * V);
  double* tl = (double*)malloc(sizeof(double) * (size_t)C * V);
  double* row = (double*)malloc(sizeof(double) * (size_t)V);
  double* q = (double*)malloc(sizeof(double) * (size_t)V);
  int32_t* prop = (int32_t*)malloc(sizeof(int32_t) * (size_t)(gamma + 1));
  int32_t* work = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + max_new + gamma + 2));
  while (len - n < max_new && rc == 0) {
    int G = gamma;
    if (C - 1 < G) G = C - 1;
    if (max_new - (len - n) < G) G = max_new - (len - n);
    if (G <= 0) break;
    memcpy(work, ids, sizeof(int32_t) * (size_t)len);
    int wl = len;
    for (int i = 0; i < G && rc == 0; i++) {
      const int t = wl < DC ? wl : DC;
      rc = oracle_forward_last_logits(draft, work + (wl - t), t, row);
      if (rc) break;
      memcpy(dl + (size_t)i * V, row, sizeof(double) * (size_t)V);
      oracle_probs_from_logits(row, V, o, q);
      prop[i] = oracle_sample_from_distribution(q, V, rng);
      work[wl++] = prop[i];
    }
    if (rc) break;
    dtok += G;
    const int ctx_len = len + G < C ? len + G : C;
    memcpy(work, ids, sizeof(int32_t) * (size_t)len);
    memcpy(work + len, prop, sizeof(int32_t) * (size_t)G);
    rc = oracle_forward(target, work + (len + G - ctx_len), ctx_len, tl);
    if (rc) break;
    calls++;
    const int base = ctx_len - G - 1;
    int acc = 0;
    const int got = oracle_speculative_round(tl + (size_t)base * V, dl, prop, G, V, max_new - (len - n), o, rng,
                                             ids + len, &acc);
    acc_total += acc;
    len += got;
  }
  if (rc == 0) memcpy(out_ids, ids, sizeof(int32_t) * (size_t)(n + max_new));
  if (stats) {
    stats[0] = calls;
    stats[1] = dtok;
    stats[2] = acc_total;
  }
  free(ids); free(dl); free(tl); free(row); free(q); free(prop); free(work);
  return rc;
}

/* FusedAttention of one sequence: the attention core of MultiHeadAttention.Forward (MultiHeadAttention.ts:46-74)
 * on given Q, K, V. ApplyRope(X, 0) (RotaryEmbedding.ts:63-75, RopeFrequencies :17-22 with base `rope_base`,
 * none when rope_base <= 0) on Q and K at positions 0..T-1, then per query head h with kv head h / (H / Hk):
 * CausalSoftmax(MatMulNT(Q_h, K_kv), 1/sqrt(d)) (CausalSoftmax.ts:17-33) @ V_kv. Row p of the result is also
 * what AttendRow (CachedRowMath.ts:60-86) gives a decode step at position p over the cached rows 0..p.
 * Layouts: q and out [T][H][d], k and v [T][Hk][d]. */
int oracle_fused_attention(const double* q, const double* k, const double* v, int T, int H, int Hk, int d,
                           double rope_base, double* out) {
  if (T < 1 || H < 1 || Hk < 1 || H % Hk != 0 || d < 2 || d % 2 != 0) return Fail("oracle_fused_attention: bad shape");
  const int G = H / Hk, half = d / 2;
  const double scale = 1.0 / sqrt((double)d);
  double* qr = (double*)malloc(sizeof(double) * (size_t)T * H * d);
  double* kr = (double*)malloc(sizeof(double) * (size_t)T * Hk * d);
  double* sc = (double*)malloc(sizeof(double) * (size_t)T);
  if (!qr || !kr || !sc) {
    free(qr);
    free(kr);
    free(sc);
    return Fail("oracle_fused_attention: out of memory");
  }
  memcpy(qr, q, sizeof(double) * (size_t)T * H * d);
  memcpy(kr, k, sizeof(double) * (size_t)T * Hk * d);
  if (rope_base > 0) {
    for (int t = 0; t < T; t++)
      for (int i = 0; i < half; i++) {
        const double ang = t * pow(rope_base, (-2.0 * i) / d);
        const double c = cos(ang), s = sin(ang);
        for (int h = 0; h < H + Hk; h++) {
          double* row = h < H ? qr + ((size_t)t * H + h) * d : kr + ((size_t)t * Hk + (h - H)) * d;
          const double x0 = row[2 * i], x1 = row[2 * i + 1];
          row[2 * i] = x0 * c - x1 * s;
          row[2 * i + 1] = x0 * s + x1 * c;
        }
      }
  }
  for (int h = 0; h < H; h++) {
    const int g = h / G;
    for (int i = 0; i < T; i++) {
      const double* qi = qr + ((size_t)i * H + h) * d;
      double mx = -INFINITY;
      for (int j = 0; j <= i; j++) {
        const double* kj = kr + ((size_t)j * Hk + g) * d;
        double dot = 0;
        for (int e = 0; e < d; e++) dot += qi[e] * kj[e];
        sc[j] = dot * scale;
        mx = fmax(mx, sc[j]);
      }
      double sum = 0;
      for (int j = 0; j <= i; j++) {
        sc[j] = exp(sc[j] - mx);
        sum += sc[j];
      }
      double* o = out + ((size_t)i * H + h) * d;
      for (int e = 0; e < d; e++) o[e] = 0;
      for (int j = 0; j <= i; j++) {
        const double w = sc[j] / sum;
        const double* vj = v + ((size_t)j * Hk + g) * d;
        for (int e = 0; e < d; e++) o[e] += w * vj[e];
      }
    }
  }
  free(qr);
  free(kr);
  free(sc);
  return 0;
}
