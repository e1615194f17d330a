/* libshahd_b200 — B200 (sm_100a) backend for the Shahd KV-cached decode path.
 *
 * A C-ABI shared library the Bun/TypeScript host loads through bun:ffi, as it loads
 * GoKernels/matmul.dll today. Two surfaces:
 *   1. the matmul-level seam of the Go FFI library (same symbol names and signatures), so the
 *      reference's GoFfiBackend loader path (Brain/ComputeBackend/GoFfiBackend.ts:92-151) works as is;
 *   2. a decode-level session API (device-resident weights, paged KV cache, batched cached steps,
 *      on-device greedy / seeded sampling) that takes over CachedDecoder / CachedGenerate.
 * All host buffers are caller-owned and only read or written during a call; the library never keeps a
 * host pointer. Device memory behind a session is owned by the session.
 *
 * Reference paths below are relative to the reference repository (Khaymah/shahd-llm-stack).
 */
#ifndef SHAHD_B200_H
#define SHAHD_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes of the int-returning entry points ------------------------------------------ */
#define SHAHD_OK 0
#define SHAHD_EINVAL (-1)   /* bad argument (the message names it, like ValidateMatMulArgs does) */
#define SHAHD_ENODEV (-2)   /* no usable sm_100 device */
#define SHAHD_ENOMEM (-3)   /* device allocation failed or KV pool exhausted */
#define SHAHD_ECUDA (-4)    /* a CUDA call failed */
#define SHAHD_ESTATE (-5)   /* call not valid in the session's current state */
#define SHAHD_ETIMEOUT (-6) /* a bounded device-side wait gave up (kernel reported it) */

/* ================================================================================================
 * 1. Matmul-level seam: drop-in for the Go FFI exports (GoKernels/ffi/matmul.go:96-118,218-395).
 *    Host pointers, row-major, i32 dims, synchronous. They return void like the Go exports; a bad
 *    argument or a device failure leaves `out` untouched and records ShahdLastError().
 * ============================================================================================== */

/* out[M,N] = a[M,K] @ b[K,N] (overwrite).                       replaces MatMulF64, matmul.go:218-235 */
void MatMulF64(const double* a, const double* b, double* out, int m, int k, int n);
/* out[M,N] (+)= a[M,K] @ btᵀ, bt stored [N,K]; acc!=0 adds.      replaces MatMulNTF64, matmul.go:242-245 */
void MatMulNTF64(const double* a, const double* bt, double* out, int m, int k, int n, int acc);
/* db[K,N] (+)= aᵀ @ dout, a [M,K], dout [M,N].                   replaces MatMulTNF64, matmul.go:252-289 */
void MatMulTNF64(const double* a, const double* dout, double* db, int m, int k, int n, int acc);
/* f32 twins.                                                     replace matmul.go:329-395
 * MatMulF32 / MatMulNTF32 with M >= 64 run on the tensor cores: operands split into two TF32 parts, three
 * tcgen05 kind::tf32 passes into fp32 accumulators (within 1e-4 of the output range); smaller M, and every
 * call while SetScalarKernels(1) is in force, run exact fp32 FMA chains on CUDA cores. MatMulTNF32 is fp32 FMA. */
void MatMulF32(const float* a, const float* b, float* out, int m, int k, int n);
void MatMulNTF32(const float* a, const float* bt, float* out, int m, int k, int n, int acc);
void MatMulTNF32(const float* a, const float* dout, float* db, int m, int k, int n, int acc);
/* Accepted for loader compatibility (matmul.go:96-99); the GPU path has no CPU fan-out to cap. */
void SetKernelThreads(int n);
/* 1 when the fast kernels can run. For this library that means a usable sm_100 device, so the
 * reference selector's probe (BackendSelector.ts:74-93, matmul.go:106-109) keeps working unchanged. */
int ShahdCpuSupportsAvx2Fma(void);
/* Test hook with the meaning of matmul.go:111-118: force != 0 makes every decode projection and the f32
 * seam run the CUDA-core (SIMT) kernels whatever the row count (exact fp32 FMA chains), so the tensor-core
 * tiles can be parity-checked against them; 0 restores the row-count rule. Process-wide. */
void SetScalarKernels(int force);

/* ---- additions of this library ---------------------------------------------------------------- */
/* 1 when device 0 is an sm_100 GPU this build can run on, else 0 (the "Gpu" slot probe,
 * BackendSelector.ts:134-137). */
int ShahdGpuAvailable(void);
/* Thread-local message of the last failure on this thread ("" when none). */
const char* ShahdLastError(void);
/* Row count from which decode projections use tcgen05 tiles instead of the SIMT kernel (default 17;
 * 1 forces tensor cores everywhere). Process-wide tuning/test hook; no counterpart in the reference. */
void ShahdSetTensorCoreMinRows(int rows);
/* Programmatic dependent launch between the kernels of a step (default 1): each kernel is scheduled
 * while its predecessor drains and overlaps its setup and weight loads. Process-wide; no counterpart in
 * the reference. */
void ShahdSetProgrammaticLaunch(int enable);
/* Concurrent chains a batched decode step is split into (independent sequences on their own streams,
 * joined in one CUDA graph); 0 = automatic (one chain). Process-wide tuning hook;
 * no counterpart in the reference. Results do not depend on it. */
void ShahdSetDecodeChains(int chains);
/* 1: greedy shahd_generate / shahd_generate_device (and shahd_generate_logits, which needs it) run every
 * decode step until the next window rebuild (or the end) in ONE persistent launch when the model fits it:
 * thread-block clusters of 16 CTAs each own up to 16 sequences for all steps (tcgen05 tiles, TMA weight
 * streaming, cluster barriers, no host round trip and no launch per step). 0 (the default, faster at the
 * shapes measured) runs one CUDA-graph-replayed launch chain per step. Results agree within the parity
 * tolerance. Process-wide; no counterpart in the reference. */
void ShahdSetPersistentStep(int enable);
/* 1 (default): causal prefill attention of head_dim 64 runs on the tensor cores (tcgen05 Q.K^T and P.V tiles
 * in TMEM, bf16 operands, fp32 softmax and accumulation); 0: the CUDA-core tile kernel (fp32 queries and
 * products). Both agree with the oracle within the parity tolerance. Process-wide; no counterpart in the
 * reference. */
void ShahdSetTensorCorePrefillAttention(int enable);
/* Decode-row attention kernel: 0 automatic (default: page streaming for rows attending >= 384 cached
 * positions on average when rows x kv heads fill the SMs, read-ahead rows otherwise), 1 the read-ahead rows
 * kernel (32-position warp tasks, K/V rows in registers), 2 the page-ring kernel (64-position pages by bulk
 * copies into a three-page ring, block-wide phases), 3 the page-streaming kernel (a producer warp's bulk
 * copies into a six-page ring, one page per compute warp, no block-wide barrier per page). Results agree
 * within the parity tolerance. Process-wide tuning hook; no counterpart in the reference. */
void ShahdSetDecodeAttentionKernel(int mode);
/* Fused decode attention block: for decode rows whose rows x kv heads fill the SMs, and models whose Q/K/V
 * rows of one kv head fit in shared memory twice per SM (head_dim 32 or 64, <= 4 query heads per kv head,
 * embedding width <= 512), 1 runs norm + Q/K/V projection + RoPE + KV append + attention + output projection
 * + residual in one launch per layer; 0 (the default) keeps the three-launch chain (QKV projection,
 * attention, O projection). Results agree within the parity tolerance. Process-wide tuning hook; no
 * counterpart in the reference. */
void ShahdSetFusedAttentionBlock(int enable);
/* Batched-prefill projections (more than 128 rows): 1 (the default) runs them on the persistent
 * warp-specialized tcgen05 kernel (TMA warp, MMA warp, eight epilogue warps, two TMEM accumulators, 128 x 256
 * or 128 x 128 tiles) after a per-row norm-statistics pass; 0 keeps one 128 x 128 tile per CTA. Results agree
 * within the parity tolerance. Process-wide tuning hook; no counterpart in the reference. */
void ShahdSetPersistentPrefillProjections(int enable);
/* First error code a kernel recorded for a bounded device-side wait that gave up (0 = none). */
int ShahdDeviceErrorFlag(void);
/* Device-pointer MatMulNT on the tensor cores: out[M,N] (+)= a[M,K] @ btᵀ with a, bt bf16 row-major
 * on the device, out fp32; tcgen05/TMEM tiles fed by TMA. K must be a multiple of 8 and the three
 * pointers 16-byte aligned. stream may be 0. Returns a status code.  (MatMulNtInto/MatMulNtAcc of
 * ComputeBackend.ts:29-36 for device-resident operands.) */
int ShahdMatMulNTBF16Device(const void* a, const void* bt, float* out, int m, int k, int n, int acc, void* stream);
/* Device-pointer MatMulNT with fp32 operands on the tensor cores: out[M,N] (+)= a[M,K] @ btᵀ, a, bt, out fp32
 * row-major on the device; the operands are split into two TF32 parts (in a per-device workspace) and
 * multiplied in three tcgen05 kind::tf32 passes with fp32 accumulation (within 1e-4 of the output range).
 * K must be a multiple of 4 and out 16-byte aligned. Asynchronous on `stream` (0 = the legacy stream); the
 * workspace is reused by the next call on the device, so calls on one device must not overlap. Returns a
 * status code.  (MatMulNtInto/MatMulNtAcc of ComputeBackend.ts:29-36 for device-resident f32 operands.) */
int ShahdMatMulNTF32Device(const float* a, const float* bt, float* out, int m, int k, int n, int acc, void* stream);
/* MatMulNTF32 that never allocates or frees device memory; no counterpart in the reference.
 * out[M,N] (+)= a[M,K] @ btᵀ with the same kernel and the same results as MatMulNTF32, but the
 * operands are staged in one fixed 16 MiB array per device that is part of the library's device image
 * instead of a workspace grown by cudaMalloc/cudaFree. For callers that cannot allocate: a process whose
 * device memory is already committed (a session KV pool sized to fill HBM), or one that must not let a
 * cudaFree wait on the whole device while other streams run decode steps.
 * Limit: 4*(round64(M*K) + round64(N*K) + M*N) <= 16 MiB; larger calls return SHAHD_EINVAL with a
 * message naming the size and the limit. The first call on each device does the set-up (looks up the
 * array's device address, which may load the library's device module): make that first call before
 * any stream capture begins. All calls on a device share the one array: calls that overlap in time
 * (from several host threads) race on it, so such callers must serialize them. Synchronous; runs on the
 * calling thread's per-thread default stream. Returns a status code. */
int ShahdMatMulNTF32NoAlloc(const float* a, const float* bt, float* out, int m, int k, int n, int acc);

/* ================================================================================================
 * 2. Decode-level session API (new surface; nothing in the reference plays this role — its decode
 *    row math is inline TS, Brain/Sampling/CachedRowMath.ts).
 * ============================================================================================== */

/* Model knobs of Brain/Config/Constants.ts:11-26 with Derived values resolved (DeriveConfig.ts:8-20). */
typedef struct ShahdModelCfg {
  int32_t embed_dim;
  int32_t num_layers;
  int32_t num_heads;
  int32_t kv_heads;        /* Derived.KvHeads (NumHeads for MHA) */
  int32_t block_size;      /* context window = KV capacity */
  int32_t vocab_size;
  int32_t mlp_hidden;      /* Derived.MlpHidden = round(EmbedDim * MlpRatio) */
  int32_t position_scheme; /* 0 = Learned, 1 = Rope */
  int32_t norm_kind;       /* 0 = LayerNorm, 1 = RmsNorm */
  int32_t mlp_kind;        /* 0 = Relu, 1 = SwiGlu, 2 = GeGlu */
  int32_t weight_tying;    /* 1 = LM head is Wteᵀ */
  int32_t reserved;        /* 0 */
  double layer_norm_eps;   /* Model.LayerNormEps */
  double rope_base;        /* RoPE theta; the reference always uses 10000 (RotaryEmbedding.ts:13) */
} ShahdModelCfg;

/* SamplingOptions (Brain/Sampling/Distribution.ts:11-15). */
typedef struct ShahdSampling {
  double temperature; /* <= 0 => greedy argmax */
  int32_t top_k;      /* 0 => disabled */
  int32_t reserved;
  double top_p;       /* 1 => disabled */
} ShahdSampling;

typedef struct ShahdSessionOpts {
  int32_t max_seqs; /* sequences held at once (slots 0..max_seqs-1) */
  int32_t kv_pages; /* KV pool size in pages of 64 positions; 0 = max_seqs * ceil(block_size / 64) */
  int32_t device;   /* CUDA device ordinal */
  int32_t flags;    /* 0 */
} ShahdSessionOpts;

typedef struct ShahdSession ShahdSession;

/* Number of parameters of Shahd.Parameters() (Brain/Nn/Shahd.ts:87-94) for cfg, or -1. */
int64_t shahd_param_count(const ShahdModelCfg* cfg);

/* The reference's weight initialization: new Shahd(Config, CreateRngStreams(seed).InitRng)
 * (Shahd.ts:30-39, InitPolicy.ts:15-24, SeededRng.ts) with InitScale 0.02 and UseScaledResidualInit,
 * written as f32 in Parameters() order. count must equal shahd_param_count(cfg). */
int shahd_init_params(const ShahdModelCfg* cfg, uint32_t seed, float* params, int64_t count);

/* Copies the parameters (Parameters() order; params_f64 = 0: float, 1: double) to the device,
 * repacked to BF16 [out,in] tiles plus fp32 norms/embeddings, and allocates the paged KV pool. */
int shahd_session_create(const ShahdModelCfg* cfg, const void* params, int32_t params_f64, int64_t params_count,
                         const ShahdSessionOpts* opts, ShahdSession** out);
int shahd_session_destroy(ShahdSession* s);

/* Forget the cached tokens of the listed slots (KvCache.Reset, KvCache.ts:62-64); frees their pages. */
int shahd_reset(ShahdSession* s, const int32_t* slots, int32_t n);
/* Cached length of one slot (KvCache.Length, KvCache.ts:52-54), or a negative status. */
int32_t shahd_seq_length(ShahdSession* s, int32_t slot);

/* PrefillCache (Brain/Sampling/CachedForward.ts:100-110) for n slots at once: slot i is reset and
 * filled with ids[offsets[i] .. offsets[i+1]) at window positions 0..len-1. offsets has n+1 entries. */
int shahd_prefill(ShahdSession* s, const int32_t* slots, const int32_t* ids, const int32_t* offsets, int32_t n);

/* CachedForwardStep (CachedForward.ts:94-96) for n slots at once: token i enters slot i at position
 * == its cached length. logits (nullable) receives [n, vocab] fp32; next_ids (nullable) receives the
 * greedy argmax of each row (ArgmaxOf, Distribution.ts:19-30). */
int shahd_step(ShahdSession* s, const int32_t* slots, const int32_t* tokens, int32_t n, float* logits,
               int32_t* next_ids);

/* CachedGenerate (CachedForward.ts:153-171) for n independent sequences, slots 0..n-1 (reset first).
 * prompts packed with offsets (n+1 entries); out_ids receives [n, max_new] new ids.
 * opts NULL or temperature <= 0: greedy (first index of the max). temperature > 0: SampleFromLogits
 * (Sampler.ts:16-27) on the device — temperature softmax, top-k, top-p over the renormalized top-k
 * mass, one SeededRng draw per new token, inverse CDF in index order (Distribution.ts:35-104).
 * rng_states [n]: SeededRng.GetState() of each sequence's sampling stream; required when
 * temperature > 0, read at entry and written back advanced by max_new draws; unused when greedy. */
int shahd_generate(ShahdSession* s, const int32_t* prompts, const int32_t* offsets, int32_t n, int32_t max_new,
                   const ShahdSampling* opts, uint32_t* rng_states, int32_t* out_ids);

/* Device-pointer twin of shahd_generate: prompts/offsets/out_ids/rng_states are device buffers and the
 * call is asynchronous on `stream` (0 = the session's stream). offsets must also be given on the host
 * (host_offsets) because the host plans pages and window slides from the lengths. */
int shahd_generate_device(ShahdSession* s, const int32_t* d_prompts, const int32_t* host_offsets, int32_t n,
                          int32_t max_new, const ShahdSampling* opts, uint32_t* d_rng_states, int32_t* d_out_ids,
                          void* stream);

/* The target pass of speculative decoding (SpeculativeDecodeGreedy, Brain/Reasoning/SpeculativeDecode.ts:
 * 67-72, with the cache instead of a full forward): slot i's tokens tokens[offsets[i] .. offsets[i+1]) are
 * appended at its cached length and the LM head runs on every appended row; next_ids [rows] receives each
 * row's greedy argmax (row j predicts the token after tokens[offsets[i] + j]) and logits (nullable)
 * [rows, vocab]. Positions must stay inside the window; at most the session's prefill chunk of rows. */
int shahd_verify(ShahdSession* s, const int32_t* slots, const int32_t* tokens, const int32_t* offsets, int32_t n,
                 float* logits, int32_t* next_ids);
/* Keep only the first lengths[i] cached positions of slot i (lengths[i] <= its length): drops the rows
 * of rejected draft tokens after a verify pass. Pages stay assigned to the slot. */
int shahd_truncate(ShahdSession* s, const int32_t* slots, const int32_t* lengths, int32_t n);

/* Greedy CachedGenerate like shahd_generate that also records every step's logits (CachedDecoder.Logits after
 * each push, CachedForward.ts:113-150): logits [n, max_new, vocab] fp32 on the host; row i, step k holds the
 * logits the id out_ids[i, k] was chosen from. Needs the persistent decode loop (greedy, a model it supports);
 * otherwise returns SHAHD_EINVAL. A parity and diagnostics entry point: the logits cross PCIe every call. */
int shahd_generate_logits(ShahdSession* s, const int32_t* prompts, const int32_t* offsets, int32_t n, int32_t max_new,
                          int32_t* out_ids, float* logits);

/* Wait for the session's outstanding device work; returns the first recorded device error, if any. */
int shahd_sync(ShahdSession* s);

/* Kernel launches of one decode step of n rows (embed, 5 per layer, head, finish). */
int32_t shahd_step_launches(ShahdSession* s, int32_t n);
/* Every kernel this session has launched so far. */
int64_t shahd_kernel_launches(ShahdSession* s);
/* Measurement hook (no counterpart in the reference): while enabled, every kernel launch of the session
 * is bracketed by CUDA events on its own stream and tagged with its class and algorithmic bytes. Steps
 * still replay as CUDA graphs (the events are event nodes of the graph, which also keeps consecutive
 * kernels from overlapping), and each step is waited for so its times can be read. Enabling (or
 * disabling) clears the totals. */
int shahd_profile(ShahdSession* s, int32_t enable);
/* Totals over the records of one class of launches: 0 = attention, 1 = projections (GEMV/GEMM incl. the LM
 * head), 2 = embed/sampler/finish of per-kernel decode steps; 3-5 = the same classes of prefill launches;
 * 6 = the persistent decode loop (one launch per run of steps). total_ms sums the launches' event times; bytes
 * sums their algorithmic bytes (weights once per step + KV rows read and written). */
int shahd_profile_read(ShahdSession* s, int32_t kind, double* total_ms, int64_t* launches, double* bytes);

/* SampleFromLogits (Sampler.ts:16-27) for `rows` independent logits rows on the current device: the
 * sampler of shahd_generate applied to caller logits [rows, vocab] (host, f32). opts NULL or
 * temperature <= 0: first index of the max, rng_states unused; else rng_states [rows] are read and
 * written back advanced by one draw each. out_ids [rows]. Synchronous. */
int shahd_sample_logits(const float* logits, int32_t rows, int32_t vocab, const ShahdSampling* opts,
                        uint32_t* rng_states, int32_t* out_ids);

/* One verification round of stochastic speculative sampling (SpeculativeSample, Brain/Reasoning/
 * SpeculativeSampling.ts:82-112) for n sequences on the current device, on caller logits (host, f32):
 * target_logits [n, gamma + 1, vocab] (row k: the target's prediction for proposal k; row g[i]: the bonus
 * position), draft_logits [n, gamma, vocab] (row k: the draft distribution proposal k was drawn from),
 * proposals [n, gamma], g [n] proposals this round (0..gamma), budget [n] new ids still allowed (>= 1).
 * Proposal k is accepted with probability min(1, p/q) (one SeededRng draw each); the first rejection is
 * replaced by a draw from the normalized max(0, p - q) (from p when that has no mass); all accepted with
 * budget left draws a bonus id from p. p and q: ProbsFromLogits with opts (temperature > 0 required).
 * out_ids [n, gamma + 1] receives the appended ids, out_count [n] their number, accepted [n] the accepted
 * proposals; rng_states [n] are read and written back advanced. Synchronous. */
int shahd_speculative_round(const float* target_logits, const float* draft_logits, const int32_t* proposals,
                            const int32_t* g, const int32_t* budget, int32_t n, int32_t gamma, int32_t vocab,
                            const ShahdSampling* opts, uint32_t* rng_states, int32_t* out_ids, int32_t* out_count,
                            int32_t* accepted);

/* ---- FusedAttention operator (MultiHeadAttention.ts:46-74 attention core + AttendRow, CachedRowMath.ts:60-86) ----
 * Causal prefill, then 1-token decode steps, on given Q, K, V over a device-resident paged cache of K (after
 * RoPE) and V rows in bf16; fp32 softmax and accumulation. num_heads query heads over kv_heads kv heads (head
 * h reads kv head h / (num_heads / kv_heads), at most 8 per kv head), head_dim 32, 64 or 128, up to
 * `capacity` positions per sequence, RoPE base rope_base (<= 0: no RoPE; pairs (2i, 2i+1) rotated by
 * position * base^(-2i/d), RotaryEmbedding.ts:17-75), scale 1/sqrt(head_dim). All Q/K/V/out pointers are
 * fp32 device memory; calls are asynchronous on `stream` (0 = the operator's own stream). Returns a status. */
typedef struct ShahdAttention ShahdAttention;
int shahd_attention_create(int32_t max_seqs, int32_t num_heads, int32_t kv_heads, int32_t head_dim, int32_t capacity,
                           double rope_base, int32_t device, ShahdAttention** out);
int shahd_attention_destroy(ShahdAttention* a);
/* Cached positions of sequence `slot` (-1 for a bad slot). */
int32_t shahd_attention_length(ShahdAttention* a, int32_t slot);
/* Sequences 0..n-1 restart at position 0: q [n, T, num_heads, d], k and v [n, T, kv_heads, d] (before RoPE);
 * out [n, T, num_heads, d] = CausalSoftmax(scale * RoPE(Q) RoPE(K)^T) V per head (CausalSoftmax.ts:17-33). */
int shahd_attention_prefill(ShahdAttention* a, const float* q, const float* k, const float* v, int32_t n, int32_t T,
                            float* out, void* stream);
/* One step for sequences 0..n-1 at their cached lengths p: q [n, num_heads, d], k and v [n, kv_heads, d] are
 * position p's rows (before RoPE); they are appended, and out [n, num_heads, d] attends over positions 0..p. */
int shahd_attention_decode(ShahdAttention* a, const float* q, const float* k, const float* v, int32_t n, float* out,
                           void* stream);
const char* shahd_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
