/* CPU oracle for the KV-cached Shahd decode path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, f64 restatement of the reference's TypeScript decode path, used by tests/ (as the
 * checker), by __graft_entry__.smoke() and by bench.py's cpu_baseline / --impl reference legs.
 * Nothing in the shipped library links, loads or calls this code.
 *
 * Parity pinning: the reference's TS/Go layers cannot run in this image (no bun, no go), so this
 * restatement is pinned by (1) the reference's own relational tests ported onto it (cached step vs
 * full forward, CachedGenerate ids == Generate ids, sliding window), (2) its literal known answers
 * (MatMulNT 2x3, identity multiply), and (3) the reference's own C matmul kernels
 * (GoKernels/ffi/matmul_*.c) compiled into oracle/_ref by oracle/Makefile.
 *
 * Every function cites the reference file:line it restates (paths relative to the reference repo).
 * JS Math.* is not bit-specified; libm exp/log/cos/sin/tanh/sqrt/pow stand in for it.
 */
#ifndef SHAHD_ORACLE_H
#define SHAHD_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Model knobs of Brain/Config/Constants.ts:11-26 plus the derived values of
 * Brain/Config/DeriveConfig.ts:8-20 (mlp_hidden is passed resolved: round(E*MlpRatio)). */
typedef struct OracleCfg {
  int32_t embed_dim;
  int32_t num_layers;
  int32_t num_heads;
  int32_t kv_heads;        /* Derived.KvHeads = KvHeads ?? NumHeads */
  int32_t block_size;
  int32_t vocab_size;
  int32_t mlp_hidden;
  int32_t position_scheme; /* 0 = Learned, 1 = Rope */
  int32_t norm_kind;       /* 0 = LayerNorm, 1 = RmsNorm */
  int32_t mlp_kind;        /* 0 = Relu, 1 = SwiGlu, 2 = GeGlu */
  int32_t weight_tying;
  int32_t use_scaled_residual_init;
  int32_t precision_f32;   /* Compute.Precision: 0 = F64, 1 = F32 tensor storage */
  int32_t pad_;
  double layer_norm_eps;
  double init_scale;
} OracleCfg;

typedef struct OracleSampling {
  double temperature; /* <= 0 => greedy */
  int32_t top_k;      /* 0 => disabled */
  int32_t pad_;
  double top_p;       /* 1 => disabled */
} OracleSampling;

/* ---- Brain/Random/SeededRng.ts ---- */
uint32_t oracle_mix_seed(uint32_t seed, uint32_t stream);           /* :7-12 */
uint32_t oracle_rng_next_u32(uint32_t* state);                      /* :32-35 */
double oracle_rng_next_float(uint32_t* state);                      /* :38-40 */
double oracle_rng_next_gaussian(uint32_t* state);                   /* :43-47 */
void oracle_create_streams(uint32_t seed, uint32_t out_states[4]);  /* :58-65 */

/* ---- parameters: flat buffer in Shahd.Parameters() order (Brain/Nn/Shahd.ts:87-94) ---- */
int64_t oracle_param_count(const OracleCfg* cfg);
/* Fills params with the reference's constructor draw order from CreateRngStreams(seed).InitRng.
 * Values are rounded to f32 when cfg->precision_f32 (Float32Array storage). */
int oracle_init_params(const OracleCfg* cfg, uint32_t seed, double* params);

/* Intra-op threads of the batched (prefill / full-forward) matmuls; results do not depend on it. */
void oracle_set_threads(int n);

/* ---- matmul semantics of the seam ---- */
void oracle_matmul(const double* a, const double* b, double* out, int m, int k, int n);       /* TsBackend.MatMul */
void oracle_matmul_nt(const double* a, const double* bt, double* out, int m, int k, int n, int acc);
void oracle_matmul_tn(const double* a, const double* dout, double* db, int m, int k, int n, int acc);

/* ---- model + KV cache ---- */
typedef struct OracleModel OracleModel;
typedef struct OracleCache OracleCache;

OracleModel* oracle_model_create(const OracleCfg* cfg, const double* params); /* copies params */
void oracle_model_destroy(OracleModel* m);
OracleCache* oracle_cache_create(const OracleModel* m);
void oracle_cache_destroy(OracleCache* c);
int oracle_cache_length(const OracleCache* c);
/* K (post-RoPE) / V rows of (layer, kv head): count*head_dim values copied into out. */
int oracle_cache_read(const OracleCache* c, int layer, int kv_head, double* k_out, double* v_out);

/* CachedForwardStep (Brain/Sampling/CachedForward.ts:94-96). Returns 0, or <0 on a validation error. */
int oracle_cached_step(const OracleModel* m, OracleCache* c, int token, int position, double* logits);
/* PrefillCache (CachedForward.ts:100-110): batched tensor forward with the KV sink. */
int oracle_prefill(const OracleModel* m, OracleCache* c, const int32_t* ids, int n);
/* Shahd.Forward (Shahd.ts:58-60): logits [T, V] of the full tensor forward. */
int oracle_forward(const OracleModel* m, const int32_t* ids, int t, double* logits);
/* Shahd.ForwardLastLogits (Shahd.ts:66-74). */
int oracle_forward_last_logits(const OracleModel* m, const int32_t* ids, int t, double* logits);

/* ---- Brain/Sampling/Distribution.ts + Sampler.ts ---- */
int oracle_argmax(const double* logits, int vocab);                                          /* :19-30 */
void oracle_probs_from_logits(const double* logits, int vocab, const OracleSampling* o, double* probs); /* :35-89 */
int oracle_sample_from_distribution(const double* probs, int vocab, uint32_t* rng_state);   /* :93-104 */
int oracle_sample_from_logits(const double* logits, int vocab, const OracleSampling* o, uint32_t* rng_state); /* Sampler.ts:16-27 */

/* ---- decode loops ---- */
/* CachedGenerate (CachedForward.ts:153-171): writes prompt_len + max_new ids into out_ids. */
int oracle_cached_generate(const OracleModel* m, const int32_t* prompt, int prompt_len, int max_new,
                           const OracleSampling* o, uint32_t* rng_state, int32_t* out_ids);
/* Generate (Generate.ts:28-43): the uncached twin. */
int oracle_generate(const OracleModel* m, const int32_t* prompt, int prompt_len, int max_new,
                    const OracleSampling* o, uint32_t* rng_state, int32_t* out_ids);
/* Independent sequences over a pthread pool (one CachedGenerate per sequence); prompts are
 * [nseq, prompt_len], out_ids [nseq, prompt_len + max_new], rng_states [nseq]. */
int oracle_cached_generate_batch(const OracleModel* m, const int32_t* prompts, int nseq, int prompt_len,
                                 int max_new, const OracleSampling* o, uint32_t* rng_states,
                                 int32_t* out_ids, int threads);

/* ---- teacher-forced decoder (CachedDecoder, CachedForward.ts:113-150) ---- */
typedef struct OracleDecoder OracleDecoder;
OracleDecoder* oracle_decoder_create(const OracleModel* m, const int32_t* prompt, int n);
int oracle_decoder_push(OracleDecoder* d, int token);
const double* oracle_decoder_logits(const OracleDecoder* d);
int oracle_decoder_cache_length(const OracleDecoder* d);
void oracle_decoder_destroy(OracleDecoder* d);

/* Teacher-forced judgement of greedy trajectories ids [nseq, nnew] produced elsewhere from prompts
 * [nseq, plen] (one CachedDecoder per sequence over a pthread pool; see oracle.c for the rule). */
int oracle_check_trajectories(const OracleModel* m, const int32_t* prompts, int nseq, int plen, const int32_t* ids,
                              int nnew, double tol, int threads, int32_t* fails, int32_t* first_fail,
                              int32_t* near_ties, double* max_gap);

/* ---- Brain/Reasoning/SpeculativeSampling.ts ---- */
/* One verification round on given logits (target [g+1][V], draft [g][V]); returns the ids appended. */
int oracle_speculative_round(const double* target, const double* draft, const int32_t* proposals, int g, int V,
                             int budget, const OracleSampling* o, uint32_t* rng, int32_t* out, int* accepted);
/* SpeculativeSample (:38-115): out_ids receives prompt + max_new ids; stats [target calls, draft tokens,
 * accepted tokens] (nullable). */
int oracle_speculative_sample(const OracleModel* target, const OracleModel* draft, const int32_t* prompt, int n,
                              int max_new, const OracleSampling* o, uint32_t* rng, int gamma, int32_t* out_ids,
                              int32_t* stats);

/* FusedAttention (MultiHeadAttention.ts:46-74 core with RoPE and CausalSoftmax) of one sequence on given Q, K,
 * V; q/out [T][H][d], k/v [T][Hk][d]; rope_base <= 0: no RoPE. Row p equals a decode step's AttendRow. */
int oracle_fused_attention(const double* q, const double* k, const double* v, int T, int H, int Hk, int d,
                           double rope_base, double* out);
const char* oracle_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
