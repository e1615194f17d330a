// Decode-level session: device-resident weights, paged KV pool, batched cached steps and the
// on-device CachedGenerate loop (Brain/Sampling/CachedForward.ts:94-199) behind the C ABI of
// include/shahd_b200.h.
//
// All device work of a session runs on the session's own stream; a caller stream passed to
// shahd_generate_device is joined with events at entry and exit. Prefill and decode steps are captured
// once per shape into CUDA graphs and replayed; positions, tokens and outputs live in device buffers, so
// a replay needs no host update.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <numeric>
#include <tuple>
#include <vector>

#include "../../include/shahd_b200.h"
#include "decode_kernels.cuh"
#include "params.h"
#include "prefill_attention.cuh"
#include "prefill_attention_umma.cuh"
#include "attn_pages.cuh"
#include "attn_block.cuh"
#include "gemm_persist.cuh"
#include "sampling.cuh"
#include "decode_loop.cuh"
#include "umma_linear.cuh"

namespace shahd {

struct Layer {
  bf16 *w_qkv, *w_o, *w_up, *w_down;
  float *qkv_c1, *qkv_c2, *up_c1, *up_c2, *b_fc, *b_proj;
};

// Everything a captured step bakes in.
struct GraphKey {
  int kind;  // 16 * (16 * steps per graph + (0 = prefill step, 1 = decode step)) + concurrent chains
  int M;
  const void *slot, *tok, *poff, *prompt, *out;
  int out_ld;
  int min_rows;
  double temperature, top_p;  // sampling knobs baked into the sampler launch (temperature 0 = greedy)
  int top_k;
  const void* logits;  // head output (verify passes run a head on prefill-style rows)
  int head;            // 2 * embed_ready of the first step + head
  int plan_i0, plan_n, plan_qblocks;  // the prefill plan entries a prefill-style step attends over
  bool operator<(const GraphKey& o) const {
    return std::tie(kind, M, slot, tok, poff, prompt, out, out_ld, min_rows, temperature, top_p, top_k, logits, head,
                    plan_i0, plan_n, plan_qblocks) <
           std::tie(o.kind, o.M, o.slot, o.tok, o.poff, o.prompt, o.out, o.out_ld, o.min_rows, o.temperature, o.top_p,
                    o.top_k, o.logits, o.head, o.plan_i0, o.plan_n, o.plan_qblocks);
  }
};

// One kernel launch bracketed by CUDA events (measurement mode).
struct ProfRec {
  int kind;
  cudaEvent_t e0, e1;
  double bytes;         // algorithmic bytes, or the part that does not grow with the cached lengths
  double per_attended;  // graph records: bytes per cached position the step's attention reads
  int chain, rep;       // which chain and which of the graph's consecutive steps the launch belongs to
};

struct StepGraph {
  cudaGraphExec_t exec;
  int launches;
  std::vector<ProfRec> recs;  // event nodes captured with the step (measurement mode only)
};

}  // namespace shahd

struct ShahdSession {
  ShahdModelCfg cfg;
  int E, L, H, Hk, d, F, C, V, G;
  int Ep, Fp, HDp;  // reduction lengths padded to multiples of 8
  int Nqkv, Nup;
  int device;
  int max_seqs;
  int rows_cap;  // rows of the activation buffers: max(max_seqs, prefill chunk)
  int num_sms;
  int chains_hint = 1;  // decode chains running concurrently (attention splits share the GPU among them)
  cudaStream_t side[7] = {};  // extra streams of the concurrent decode chains
  cudaEvent_t fork_ev = nullptr, chain_ev[7] = {};
  cudaStream_t stream = nullptr;
  cudaEvent_t join_in = nullptr, join_out = nullptr;
  std::mutex mu;
  std::vector<void*> allocs;
  std::map<void*, size_t> alloc_bytes;

  std::vector<shahd::Layer> layers;
  shahd::bf16* w_head;
  float *head_bias, *head_c1, *head_c2, *wte, *wpe, *rope_cos, *rope_sin;

  // paged KV pool
  shahd::bf16* kv_pool;
  size_t page_elems;
  int kv_pages, max_blocks;
  int* d_block_table;
  int* h_block_table = nullptr;  // pinned mirror
  CUtensorMap kv_tmap;     // the pool as rows of d dims (head_dim 64): TMA source of the tensor-core prefill attention
  bool kv_tmap_ok = false;
  std::vector<int> free_pages;
  std::vector<int> h_len;
  int* d_seq_len;

  // per-row scratch (capacity max_seqs rows): fp32 masters and bf16 tensor-core operands
  float *x, *q, *ctx, *act, *logits, *am_val;
  shahd::bf16 *xb, *ctxb, *actb;
  int* am_idx;
  int am_stride;
  float *part_o, *part_m, *part_l;
  int* attn_counter;
  float* row_stats = nullptr;  // [rows_cap][2] norm statistics of the prefill rows (persistent projections)
  bool ab_ok = false;  // the model's shape fits the fused attention block (one kv head's weights next to a second CTA)
  // persistent cluster decode loop: weight tensor maps (box 64 x 128) and per-layer constants in device memory
  int loop_state = -1;  // -1 not set up yet, 0 unavailable for this model/device, 1 ready
  shahd::LoopLayer* d_loop_layers = nullptr;
  std::vector<CUtensorMap> loop_wmaps;  // copied into every launch's parameters
  int loop_max_clusters = 0;  // clusters of kLoopCS CTAs resident at once with the loop's shared memory
  float* d_loop_logits = nullptr;  // recorded logits of shahd_generate_logits [rows, steps, V]
  size_t loop_logits_cap = 0;
  unsigned long long* d_loop_trace = nullptr;  // per-phase timestamps when SHAHD_LOOP_TRACE names a file
  size_t loop_trace_cap = 0;
  // verify passes (speculative decoding): per-row logits, argmax partials and ids, grown on demand
  float* d_vlogits = nullptr;
  float* d_vam_val = nullptr;
  int* d_vam_idx = nullptr;
  int* d_vids = nullptr;
  int vrows_cap = 0;
  // split-K partial tiles of the norm-free projections, one region per decode chain
  float* split_ws;
  int* split_cnt;
  size_t split_ws_floats;
  int split_cnt_len;
  int *d_slot, *d_tok, *d_pos, *d_next, *d_gen_count, *d_ends, *d_starts, *d_full_len, *d_rows;
  uint32_t* d_rng;  // [max_seqs] SeededRng state per slot while a stochastic generate runs
  int* d_sampled;   // [max_seqs] ids the sampler chose this step
  int *d_seq_plan;                              // [5][max_seqs]: slot, token start, length, row offset, base position
  int *d_row_slot, *d_row_pos, *d_row_poff;     // [rows_cap] expanded prefill rows
  int* d_prompt = nullptr;
  size_t prompt_cap = 0;
  int* d_window;
  int* d_out = nullptr;
  size_t out_cap = 0;
  int* h_pinned_rows = nullptr;  // pinned staging for per-call row arrays [kStagingRows][max_seqs]

  std::map<shahd::GraphKey, shahd::StepGraph> graphs;

  // measurement: kernel launch count, and optional CUDA-event timing per kernel class
  long long launches = 0;
  bool prof = false;
  bool capturing = false;
  int cur_rep = 0;  // which of a graph's consecutive steps is being enqueued
  std::vector<cudaEvent_t> ev_pool;       // eager launches (recycled after each harvest)
  size_t ev_used = 0;
  std::vector<cudaEvent_t> graph_events;  // owned by captured graphs
  std::vector<shahd::ProfRec> prof_recs;  // eager records not yet harvested
  double prof_ms[7] = {}, prof_bytes[7] = {};
  long long prof_n[7] = {};
};

namespace shahd {

namespace {

// Pinned staging rows (each max_seqs ints). A row is rewritten only after the stream has drained the
// copies that read it, so no two uses between two stream synchronizations may share a row:
// 0-1 per-call slots/tokens (or a generate's RNG states), 2-5 generate plan, 6 window-rebuild rows,
// 7 lengths, 8-12 the prefill plan.
constexpr int kStagingRows = 13;
constexpr int kStagingLengths = 7;
constexpr int kPrefillRows = 8192;  // rows of one batched prefill chunk (whole sequences per chunk)
constexpr int kMaxChains = 8;
constexpr int kStepsPerGraph = 8;  // decode steps captured back to back in one graph

template <class T>
int DevAlloc(ShahdSession* s, T** p, size_t count) {
  void* v = nullptr;
  if (count == 0) count = 1;
  cudaError_t e = cudaMalloc(&v, count * sizeof(T));
  if (e != cudaSuccess) {
    SetError("cudaMalloc of %zu bytes failed: %s", count * sizeof(T), cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? SHAHD_ENOMEM : SHAHD_ECUDA;
  }
  s->allocs.push_back(v);
  s->alloc_bytes[v] = count * sizeof(T);
  *p = static_cast<T*>(v);
  return SHAHD_OK;
}

#define SHAHD_TRY(expr)              \
  do {                               \
    int rc_ = (expr);                \
    if (rc_ != SHAHD_OK) return rc_; \
  } while (0)

// ---- linear launcher: SIMT (few rows) or tcgen05 tiles (batched rows) ----------------------------

template <int MT, int NORM, class Epi>
void LaunchSimt(const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  const size_t smem = (size_t)MT * la.Kp * sizeof(float);
  if (!EnsureKernelAttrs((const void*)LinearSimtKernel<MT, NORM, Epi>, 224 * 1024)) return;
  dim3 grid(CeilDiv(la.N, kSimtCols), CeilDiv(la.M, MT));
  LaunchPdl(LinearSimtKernel<MT, NORM, Epi>, grid, dim3(kSimtWarps * 32), smem, st, la, epi);
}

template <int NORM, class Epi>
void LaunchLinearNorm(const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  if constexpr (PersistUsed<NORM, Epi>::value) {
    // batched prefill rows: the persistent warp-specialized kernel (norm statistics precomputed)
    if (g_persist_linear && la.M > kUmmaBM && la.M >= kUmmaMinRows && UmmaLinearSupported(la) &&
        (NORM == kNormNone || la.stats != nullptr)) {
      LaunchPersistLinear<NORM, Epi>(la, epi, st);
      return;
    }
  }
  if (la.M >= kUmmaMinRows && UmmaLinearSupported(la)) {
    LaunchUmmaLinear<NORM, Epi>(la, epi, st);
  } else if (la.M <= 1) {
    LaunchSimt<1, NORM, Epi>(la, epi, st);
  } else if (la.M <= 4) {
    LaunchSimt<4, NORM, Epi>(la, epi, st);
  } else {
    LaunchSimt<16, NORM, Epi>(la, epi, st);
  }
}

template <class Epi>
void LaunchLinear(int norm, const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  if (norm == kNormRms) LaunchLinearNorm<kNormRms, Epi>(la, epi, st);
  else if (norm == kNormLayer) LaunchLinearNorm<kNormLayer, Epi>(la, epi, st);
  else LaunchLinearNorm<kNormNone, Epi>(la, epi, st);
}

void LaunchRowStats(const float* x, int ldx, int K, int M, int norm, float eps, float* stats, cudaStream_t st) {
  LaunchPdl(RowStatsKernel, dim3(CeilDiv(M, 8)), dim3(256), 0, st, x, ldx, K, M, norm, eps, stats);
}

// Number of argmax partial blocks the head launch produces per row.
int HeadBlocks(const ShahdSession* s, int M) {
  LinearArgs la{};
  la.M = M;
  la.K = s->E;
  la.Kp = s->Ep;
  la.N = s->V;
  la.ab = s->xb;
  if (M >= kUmmaMinRows && UmmaLinearSupported(la)) return CeilDiv(la.N, UmmaBN(M, la.N));
  return CeilDiv(s->V, kSimtCols);
}

struct StepPlan {
  int M;
  const int* pos_in; // device [M] explicit positions (batched prefill rows) or nullptr: the slots' lengths
  bool finish;       // run the finish kernel (lengths advance, greedy id); off for batched prefill
  const int* slot;   // device [M]
  const int* tok;    // device [M] (direct tokens) or nullptr
  const int* poff;   // device [M] prompt gather offsets, or nullptr
  const int* prompt; // device packed ids for the gather
  bool head;         // run final norm + LM head + argmax
  float* logits;     // device [M, V] or nullptr
  int* next_ids;     // device [M] or nullptr
  int* cur_tok;      // device [M] or nullptr
  int* out_ids;      // device [M, out_ld] or nullptr
  int out_ld;
  long long attended;  // sum over rows of (position + 1): cached positions the attention reads
  ShahdSampling sampling;  // temperature > 0: seeded sampling from `logits` instead of the greedy argmax
  float* am_val = nullptr;  // argmax partials of a head over more rows than max_seqs (verify passes)
  int* am_idx = nullptr;
  bool embed_ready = false;  // x, xb and positions already hold this step's input (previous finish kernel)
  // prefill-style chunks: the chunk's sequences as entries plan_i0 .. plan_i0 + plan_n - 1 of the prefill
  // plan, for the tiled causal attention (plan_qblocks = 64-query blocks of the longest sequence)
  const int* seq_plan = nullptr;
  int plan_i0 = 0, plan_n = 0, plan_qblocks = 0;
  long long kv_streamed = 0;  // cached positions the tiled kernel reads: per sequence and query block, keys 0 .. last query
};

// ---- measurement hooks: kernel classes timed with CUDA events on the launching stream ---------------
// Classes 0-2 are decode-step launches; prefill launches (steps without the finish kernel) land in 3-5.
// Class 6: the persistent cluster decode loop (every decode step of a run in one launch).
enum ProfKind { kProfAttention = 0, kProfLinear = 1, kProfOther = 2, kProfPrefill = 3, kProfLoop = 6, kProfKinds = 7 };

// An event recorded on `st`: inside a stream capture it becomes an event-record node of the graph (each
// replay records it again), otherwise a plain record from the recycled pool.
cudaEvent_t ProfEvent(ShahdSession* s, cudaStream_t st) {
  cudaEvent_t e = nullptr;
  if (s->capturing) {
    cudaEventCreate(&e);
    s->graph_events.push_back(e);
    cudaEventRecordWithFlags(e, st, cudaEventRecordExternal);
    return e;
  }
  if (s->ev_used == s->ev_pool.size()) {
    cudaEventCreate(&e);
    s->ev_pool.push_back(e);
  }
  e = s->ev_pool[s->ev_used++];
  cudaEventRecord(e, st);
  return e;
}

// `bytes` is the launch's algorithmic traffic; an attention launch also passes the part that grows with
// the cached lengths (per_attended x attended) so a replayed graph can be charged for the lengths of the
// step it replays.
template <class F>
void Timed(ShahdSession* s, cudaStream_t st, int kind, double bytes, F&& launch, double per_attended = 0,
           double attended = 0, int chain = 0) {
  s->launches++;
  if (!s->prof) {
    launch();
    return;
  }
  const cudaEvent_t e0 = ProfEvent(s, st);
  launch();
  const cudaEvent_t e1 = ProfEvent(s, st);
  if (s->capturing) s->prof_recs.push_back({kind, e0, e1, bytes, per_attended, chain, s->cur_rep});
  else s->prof_recs.push_back({kind, e0, e1, bytes + per_attended * attended, 0.0, chain, 0});
}

template <int D, int NW>
void LaunchAttnRowsDW(int G, dim3 grid, cudaStream_t st, const AttnArgs& aa) {
  const int sm = AttnRowsSmem(G, D);
  if (G == 1) LaunchPdl(AttnRowsKernel<D, 1, NW>, grid, dim3(NW * 32), sm, st, aa);
  else if (G == 2) LaunchPdl(AttnRowsKernel<D, 2, NW>, grid, dim3(NW * 32), sm, st, aa);
  else if (G <= 4) LaunchPdl(AttnRowsKernel<D, 4, NW>, grid, dim3(NW * 32), sm, st, aa);
  else LaunchPdl(AttnRowsKernel<D, 8, NW>, grid, dim3(NW * 32), sm, st, aa);
}

// Decode-row attention for head_dim d in {32, 64, 128} and G <= kMaxGroup query heads per kv head:
// 8-warp CTAs while the grid fits two per SM, 4-warp CTAs beyond.
void LaunchAttnRows(int d, int G, dim3 grid, int num_sms, cudaStream_t st, const AttnArgs& aa) {
  const bool wide = (long long)grid.x * grid.y * grid.z <= 2LL * num_sms;
  if (d == 64) (wide ? LaunchAttnRowsDW<64, 8> : LaunchAttnRowsDW<64, 4>)(G, grid, st, aa);
  else if (d == 32) (wide ? LaunchAttnRowsDW<32, 8> : LaunchAttnRowsDW<32, 4>)(G, grid, st, aa);
  else (wide ? LaunchAttnRowsDW<128, 8> : LaunchAttnRowsDW<128, 4>)(G, grid, st, aa);
}

template <int D>
void LaunchAttnPagesD(int G, dim3 grid, cudaStream_t st, const AttnArgs& aa) {
  if (G == 1) LaunchPdl(AttnPagesKernel<D, 1>, grid, dim3(kApThreads), ApSmemBytes(D, 1), st, aa);
  else if (G == 2) LaunchPdl(AttnPagesKernel<D, 2>, grid, dim3(kApThreads), ApSmemBytes(D, 2), st, aa);
  else if (G <= 4) LaunchPdl(AttnPagesKernel<D, 4>, grid, dim3(kApThreads), ApSmemBytes(D, 4), st, aa);
  else LaunchPdl(AttnPagesKernel<D, 8>, grid, dim3(kApThreads), ApSmemBytes(D, 8), st, aa);
}

// Decode-row attention streaming 64-position pages (head_dim 32, 64 or 128, G <= kMaxGroup).
void LaunchAttnPages(int d, int G, dim3 grid, cudaStream_t st, const AttnArgs& aa) {
  if (d == 64) LaunchAttnPagesD<64>(G, grid, st, aa);
  else if (d == 32) LaunchAttnPagesD<32>(G, grid, st, aa);
  else LaunchAttnPagesD<128>(G, grid, st, aa);
}

template <int D>
bool EnsureAttnPagesAttrs() {
  return EnsureKernelAttrs((const void*)AttnPagesKernel<D, 1>, ApSmemBytes(D, 1)) &&
         EnsureKernelAttrs((const void*)AttnPagesKernel<D, 2>, ApSmemBytes(D, 2)) &&
         EnsureKernelAttrs((const void*)AttnPagesKernel<D, 4>, ApSmemBytes(D, 4)) &&
         EnsureKernelAttrs((const void*)AttnPagesKernel<D, 8>, ApSmemBytes(D, 8));
}

// A prefill-style step whose attention runs as query-block tiles (PrefillAttnKernel) rather than per row.
bool PrefillTiled(const ShahdSession* s, const StepPlan& p) {
  return p.seq_plan != nullptr && p.plan_n > 0 && s->G <= kPfMaxG && (s->d == 32 || s->d == 64 || s->d == 128);
}

// Cached positions an attention launch of plan p reads per kv head and layer.
double AttendedPositions(const ShahdSession* s, const StepPlan& p) {
  return (double)(PrefillTiled(s, p) ? p.kv_streamed : p.attended);
}

// Adds the event times of finished records to the per-class totals (the stream must be idle). plans
// (graph replays) give the cached lengths of the replayed steps: rep j of a chain attends j more
// positions per row than its first step.
int Accumulate(ShahdSession* s, const std::vector<ProfRec>& recs, const StepPlan* plans = nullptr) {
  for (const auto& r : recs) {
    float t = 0;
    SHAHD_CUDA_TRY(cudaEventElapsedTime(&t, r.e0, r.e1));
    double b = r.bytes;
    if (plans && r.per_attended > 0)
      b += r.per_attended * (AttendedPositions(s, plans[r.chain]) + (double)r.rep * plans[r.chain].M);
    s->prof_ms[r.kind] += t;
    s->prof_bytes[r.kind] += b;
    s->prof_n[r.kind] += 1;
  }
  return SHAHD_OK;
}

int HarvestEager(ShahdSession* s) {
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  SHAHD_TRY(Accumulate(s, s->prof_recs));
  s->prof_recs.clear();
  s->ev_used = 0;
  return SHAHD_OK;
}

// Algorithmic bytes of one projection: bf16 weights once, bf16 activations in, fp32 results out.
double LinearBytes(int M, int K, int Kp, int N) { return 2.0 * N * Kp + 2.0 * M * K + 4.0 * M * N; }

LinearArgs Lin(const float* a, int lda, const bf16* ab, int ldab, int rows_cap, int M, int K, int Kp, const bf16* w,
               int N, float eps, const float* c1, const float* c2, float* amv = nullptr, int* ami = nullptr) {
  LinearArgs la{};
  la.a = a; la.lda = lda; la.ab = ab; la.ldab = ldab; la.a_rows = rows_cap; la.M = M; la.K = K; la.Kp = Kp;
  la.w = w; la.N = N; la.eps = eps; la.c1 = c1; la.c2 = c2; la.am_val = amv; la.am_idx = ami;
  la.ws = nullptr; la.ws_cnt = nullptr;
  return la;
}

// Whether a step's finish kernel also embeds the next step's input (decode-loop steps), so that the
// following step skips its embed kernel.
bool EmbedsNext(const StepPlan& p) {
  return p.finish && p.head && p.cur_tok != nullptr && p.out_ids != nullptr;
}

// Position splits per (decode row, kv head) of the read-ahead rows kernel: enough CTAs to fill the GPU when
// the rows and kv heads alone leave SMs idle, one split otherwise (and beyond max_seqs rows).
int RowSplits(const ShahdSession* s, int M, int r0) {
  if (r0 + M <= s->max_seqs && M * s->Hk < s->num_sms)
    return std::max(1, std::min(s->max_blocks, CeilDiv(2 * s->num_sms / std::max(1, s->chains_hint), M * s->Hk)));
  return 1;
}

// Whether a decode step of M rows (rows [r0, r0 + M)) runs the fused attention block: it is switched on, the
// model fits it, the rows and kv heads fill the SMs with one CTA each, and the decode attention kernel is left
// automatic (or set to the read-ahead rows kernel, whose task layout the block shares).
bool UsesFusedBlock(const ShahdSession* s, int M, int r0) {
  return s->ab_ok && g_fused_attn_block && g_decode_attn_kernel <= 1 && r0 + M <= s->max_seqs &&
         RowSplits(s, M, r0) == 1;
}

// Enqueue one batched cached step (AdvanceOneToken + HeadLogitsRow for M rows) on `st`; returns the
// number of kernels it launched.
int EnqueueStep(ShahdSession* s, const StepPlan& p, cudaStream_t st, int r0 = 0, int chain = 0) {
  // Row-indexed buffers: activations and positions hold rows_cap rows, the LM-head / finish / attention
  // split scratch holds max_seqs rows. This step uses rows [r0, r0 + M) of them (a decode chain's window).
  // A step beyond either is a caller bug, not a device fault.
  if (p.M < 1 || r0 < 0 || r0 + p.M > s->rows_cap ||
      ((p.finish || (p.head && p.am_val == nullptr)) && r0 + p.M > s->max_seqs)) {
    SetError("internal: step of rows [%d, %d) exceeds the session's row buffers", r0, r0 + p.M);
    return -1;
  }
  const long long before = s->launches;
  const int M = p.M, R = s->rows_cap - r0;  // R: rows addressable from the window base (TMA map height)
  const int pk = p.finish ? 0 : kProfPrefill;  // measurement class offset: decode step or prefill
  const int norm = s->cfg.norm_kind == 1 ? kNormRms : kNormLayer;
  const float eps = (float)s->cfg.layer_norm_eps;
  const int hd = s->H * s->d;
  float* x = s->x + (size_t)r0 * s->E;
  bf16* xb = s->xb + (size_t)r0 * s->Ep;
  float* q = s->q + (size_t)r0 * hd;
  float* ctx = s->ctx + (size_t)r0 * hd;
  bf16* ctxb = s->ctxb + (size_t)r0 * s->HDp;
  float* act = s->act + (size_t)r0 * s->F;
  bf16* actb = s->actb + (size_t)r0 * s->Fp;
  int* pos = s->d_pos + r0;
  // scratch that exists for decode rows only (r0 + M <= max_seqs when used)
  const size_t rd = (size_t)std::min(r0, s->max_seqs);
  float* am_val = p.am_val ? p.am_val : s->am_val + rd * s->am_stride;
  int* am_idx = p.am_idx ? p.am_idx : s->am_idx + rd * s->am_stride;
  int* gen_count = s->d_gen_count + rd;
  float* part_o = s->part_o + rd * s->H * s->max_blocks * s->d;
  float* part_m = s->part_m + rd * s->H * s->max_blocks;
  float* part_l = s->part_l + rd * s->H * s->max_blocks;
  int* counter = s->attn_counter + rd * s->Hk;
  float* split_ws = s->split_ws + (size_t)chain * s->split_ws_floats;
  int* split_cnt = s->split_cnt + (size_t)chain * s->split_cnt_len;
  int nblk = 0;
  {
    if (!p.embed_ready) {
      Timed(s, st, pk + kProfOther, 8.0 * M * s->E, [&] {
        EmbedArgs e{p.pos_in, p.slot, p.tok, p.prompt, p.poff, s->d_seq_len, pos, s->wte, s->wpe, x, xb, s->E, s->Ep};
        LaunchPdl(EmbedKernel, dim3(M), dim3(128), 0, st, e);
      });
    }
    KvView kv{s->kv_pool, s->d_block_table, s->max_blocks, s->Hk, s->d, s->page_elems};
    // the fp32 context and MLP activation rows feed only the CUDA-core projections (few rows); the
    // tensor-core projections read the bf16 copies, so the fp32 rows are not written for them
    const bool tc_rows = M >= kUmmaMinRows;
    float* ctx_f32 = tc_rows ? nullptr : ctx;
    float* act_f32 = tc_rows ? nullptr : act;
    // K and V rows read (bf16) + q read and ctx written (bf16, and fp32 for the CUDA-core projection)
    const double attn_fixed = (tc_rows ? 6.0 : 10.0) * M * hd, attn_per_pos = 4.0 * s->Hk * s->d;
    // splits per (row, kv head): enough CTAs to fill the GPU; one split (no partials) beyond max_seqs rows
    int nsplit = 1;
    if (r0 + M <= s->max_seqs)
      nsplit = std::max(1, std::min(s->max_blocks, CeilDiv(3 * s->num_sms / std::max(1, s->chains_hint), M * s->Hk)));
    // decode rows (one appended position per row, distinct slots): the read-ahead kernel, split only when
    // the rows and kv heads alone leave the SMs idle
    // decode rows (one appended position per row): long cached lengths over a grid that fills the GPU go to
    // the page-streaming kernel, the rest to the read-ahead rows kernel
    const bool dec_rows = p.pos_in == nullptr && s->G <= kMaxGroup && (s->d == 32 || s->d == 64 || s->d == 128);
    const bool long_rows = (double)p.attended >= (double)kApMinMeanLen * M && M * s->Hk >= s->num_sms;
    const bool pages_kernel = dec_rows && (g_decode_attn_kernel == 3 || (g_decode_attn_kernel == 0 && long_rows));
    const bool rows_kernel = dec_rows && !pages_kernel && g_decode_attn_kernel != 2;
    const int rsplit = RowSplits(s, M, r0);
    // batched prefill rows: norm-consuming projections on the persistent kernel after a row-statistics pass
    const bool persist = g_persist_linear && M > kUmmaBM && M >= kUmmaMinRows;
    float* stats = s->row_stats + 2 * (size_t)r0;
    // decode rows that fill the SMs without position splits (any cached length): the attention half of each
    // layer in one launch
    const bool fused_block = dec_rows && UsesFusedBlock(s, M, r0);
    for (int l = 0; l < s->L; l++) {
      const Layer& Ly = s->layers[l];
      if (fused_block) {
        // norm1 + QKV + RoPE + KV append + attention + summed per-head Wo + residual (CachedForward.ts:66-84).
        // Layer 0 follows the embed / finish kernel, which writes the rows' positions: it reads them (and the
        // cached rows) after the grid-dependency wait; later layers follow the MLP and read ahead.
        const AttnBlockArgs ab{x, xb, s->E, s->Ep, s->Ep, Ly.qkv_c1, Ly.qkv_c2, norm, eps, Ly.w_o, s->HDp,
                               s->rope_cos, s->rope_sin, kv, l, pos, p.slot, s->H, s->Hk, s->G,
                               (float)(1.0 / std::sqrt((double)s->d)), l > 0 ? 1 : 0};
        const double wbytes = LinearBytes(M, s->E, s->Ep, s->Nqkv) + LinearBytes(M, hd, s->HDp, s->E);
        Timed(s, st, pk + kProfAttention, attn_fixed + wbytes,
              [&] { LaunchAttnBlock(s->d, ab, Ly.w_qkv, s->Nqkv, M, st); }, attn_per_pos, AttendedPositions(s, p),
              chain);
      } else {
        // norm1 + QKV + RoPE + KV append (CachedForward.ts:66-73, :78-79)
        LinearArgs la = Lin(x, s->E, xb, s->Ep, R, M, s->E, s->Ep, Ly.w_qkv, s->Nqkv, eps, Ly.qkv_c1, Ly.qkv_c2);
        if (persist) {
          Timed(s, st, pk + kProfLinear, 8.0 * M * s->E, [&] { LaunchRowStats(x, s->E, s->E, M, norm, eps, stats, st); });
          la.stats = stats;
        }
        const EpiQKV eq{q, kv, l, pos, p.slot, s->rope_cos, s->rope_sin, s->H, s->Hk, s->d};
        Timed(s, st, pk + kProfLinear, LinearBytes(M, s->E, s->Ep, s->Nqkv), [&] { LaunchLinear(norm, la, eq, st); });
        // attention over the cache (CachedForward.ts:76-80)
        AttnArgs aa{q, ctx_f32, ctxb, s->HDp, kv, l, pos, p.slot, s->H, s->Hk, s->G, s->d,
                    (float)(1.0 / std::sqrt((double)s->d)), s->max_blocks, part_o, part_m, part_l, counter};
        dim3 ag(nsplit, s->Hk, M);
        const bool tiled = PrefillTiled(s, p);
        const PrefillAttnArgs pa{q, ctx_f32, ctxb, s->HDp, kv, l, s->H, s->Hk, s->G,
                                 (float)(1.0 / std::sqrt((double)s->d)), p.seq_plan, s->max_seqs, p.plan_i0};
        const dim3 pg(p.plan_qblocks, s->Hk, p.plan_n);
        Timed(s, st, pk + kProfAttention, attn_fixed, [&] {
          if (pages_kernel) {
            LaunchAttnPages(s->d, s->G, ag, st, aa);
          } else if (rows_kernel) {
            LaunchAttnRows(s->d, s->G, dim3(rsplit, s->Hk, M), s->num_sms, st, aa);
          } else if (tiled && s->d == kFaD && g_umma_prefill_attn && s->kv_tmap_ok) {
            const FaArgs fa{s->kv_tmap, pa, s->L, CeilDiv(p.plan_qblocks * kPfQ, kFaQ)};
            LaunchPdl(PrefillAttnUmmaKernel, dim3(fa.qblocks, s->H, p.plan_n), dim3(kFaThreads), kFaSmemLaunch, st, fa);
          } else if (tiled) {
            if (s->d == 64) LaunchPdl(PrefillAttnKernel<64>, pg, dim3(kPfThreads), PrefillAttnSmem(64), st, pa);
            else if (s->d == 32) LaunchPdl(PrefillAttnKernel<32>, pg, dim3(kPfThreads), PrefillAttnSmem(32), st, pa);
            else LaunchPdl(PrefillAttnKernel<128>, pg, dim3(kPfThreads), PrefillAttnSmem(128), st, pa);
          } else if (s->d == 64) LaunchPdl(AttnDecodeKernel<64>, ag, dim3(kAttnThreads), AttnSmemBytes(64), st, aa);
          else if (s->d == 32) LaunchPdl(AttnDecodeKernel<32>, ag, dim3(kAttnThreads), AttnSmemBytes(32), st, aa);
          else if (s->d == 128) LaunchPdl(AttnDecodeKernel<128>, ag, dim3(kAttnThreads), AttnSmemBytes(128), st, aa);
          else LaunchPdl(AttnDecodeGenericKernel, ag, dim3(kAttnThreads), 0, st, aa);
        }, attn_per_pos, AttendedPositions(s, p), chain);
        // summed per-head Wo + residual (CachedForward.ts:81-84)
        LinearArgs lo = Lin(ctx, hd, ctxb, s->HDp, R, M, hd, s->HDp, Ly.w_o, s->E, eps, nullptr, nullptr);
        lo.ws = split_ws;
        lo.ws_cnt = split_cnt;
        Timed(s, st, pk + kProfLinear, LinearBytes(M, hd, s->HDp, s->E),
              [&] { LaunchLinear(kNormNone, lo, EpiResid{x, xb, s->E, s->Ep, nullptr}, st); });
      }
      // norm2 + MLP + residual (CachedForward.ts:86-87)
      LinearArgs lu = Lin(x, s->E, xb, s->Ep, R, M, s->E, s->Ep, Ly.w_up, s->Nup, eps, Ly.up_c1, Ly.up_c2);
      if (persist) {
        Timed(s, st, pk + kProfLinear, 8.0 * M * s->E, [&] { LaunchRowStats(x, s->E, s->E, M, norm, eps, stats, st); });
        lu.stats = stats;
      }
      Timed(s, st, pk + kProfLinear, LinearBytes(M, s->E, s->Ep, s->Nup), [&] {
        if (s->cfg.mlp_kind == 0) LaunchLinear(norm, lu, EpiReluFc{act, actb, s->F, s->Fp, Ly.b_fc}, st);
        else LaunchLinear(norm, lu, EpiGated{act_f32, actb, s->F, s->Fp, s->cfg.mlp_kind == 2}, st);
      });
      LinearArgs ld = Lin(act, s->F, actb, s->Fp, R, M, s->F, s->Fp, Ly.w_down, s->E, eps, nullptr, nullptr);
      ld.ws = split_ws;
      ld.ws_cnt = split_cnt;
      Timed(s, st, pk + kProfLinear, LinearBytes(M, s->F, s->Fp, s->E),
            [&] { LaunchLinear(kNormNone, ld, EpiResid{x, xb, s->E, s->Ep, Ly.b_proj}, st); });
    }
    if (p.head) {
      // final norm + LM head + argmax partials (HeadLogitsRow, CachedRowMath.ts:117-137)
      nblk = HeadBlocks(s, M);
      const LinearArgs lh = Lin(x, s->E, xb, s->Ep, R, M, s->E, s->Ep, s->w_head, s->V, eps, s->head_c1,
                                s->head_c2, am_val, am_idx);
      Timed(s, st, pk + kProfLinear, LinearBytes(M, s->E, s->Ep, s->V),
            [&] { LaunchLinear(norm, lh, EpiLogits{p.logits, s->head_bias, s->V}, st); });
    }
  }
  int* sampled = nullptr;
  if (p.head && p.finish && p.sampling.temperature > 0) {
    // SampleFromLogits with Temperature > 0 (Sampler.ts:16-27): one CTA per row over its logits
    sampled = s->d_sampled + rd;
    const SampleArgs sa{p.logits, s->V, p.slot, s->d_rng, (float)p.sampling.temperature, p.sampling.top_k,
                        p.sampling.top_p, sampled};
    Timed(s, st, pk + kProfOther, 4.0 * M * s->V,
          [&] { LaunchPdl(SampleKernel, dim3(M), dim3(kSampleThreads), 0, st, sa); });
  }
  if (p.finish) {
    FinishArgs f{M, p.slot, pos, s->d_seq_len, p.head ? am_val : nullptr, am_idx, nblk, p.next_ids,
                 p.cur_tok, p.out_ids, p.out_ld, gen_count, sampled, nullptr, nullptr, nullptr, nullptr,
                 s->E, s->Ep, s->C};
    if (EmbedsNext(p)) {
      f.wte = s->wte;
      f.wpe = s->wpe;
      f.x = x;
      f.xb = xb;
    }
    Timed(s, st, pk + kProfOther, 16.0 * M, [&] { LaunchPdl(FinishKernel, dim3(CeilDiv(M, 4)), dim3(128), 0, st, f); });
  }
  return (int)(s->launches - before);
}

// Concurrent decode chains for n rows: the process-wide setting, else one chain (measured: a step's time
// is its serial kernel latency, which splitting the rows does not shorten).
int DecodeChains(int n) {
  int c = g_decode_chains > 0 ? g_decode_chains : 1;
  return std::max(1, std::min(std::min(c, kMaxChains), n));
}

// Reports a kernel that failed to launch (or could not be prepared) since the last check, then any sticky
// runtime error.
int CheckLaunch(const char* what) {
  std::string where;
  cudaError_t e = TakeLaunchError(&where);
  if (e != cudaSuccess) {
    cudaGetLastError();
    SetError("%s: %s failed: %s", what, where.c_str(), cudaGetErrorString(e));
    return SHAHD_ECUDA;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    SetError("%s: kernel launch failed: %s", what, cudaGetErrorString(e));
    return SHAHD_ECUDA;
  }
  return SHAHD_OK;
}

// Enqueue several steps as concurrent chains: chain c runs on its own stream over its own row window
// (r0[c]), forked from and joined back into the session stream with events. Returns the kernels launched.
int EnqueueChains(ShahdSession* s, const StepPlan* plans, const int* r0, int nchain) {
  int total = 0;
  if (nchain > 1) {
    cudaEventRecord(s->fork_ev, s->stream);
    for (int c = 1; c < nchain; c++) cudaStreamWaitEvent(s->side[c - 1], s->fork_ev, 0);
  }
  for (int c = 0; c < nchain; c++) total += EnqueueStep(s, plans[c], c == 0 ? s->stream : s->side[c - 1], r0[c], c);
  if (nchain > 1) {
    for (int c = 1; c < nchain; c++) {
      cudaEventRecord(s->chain_ev[c - 1], s->side[c - 1]);
      cudaStreamWaitEvent(s->stream, s->chain_ev[c - 1], 0);
    }
  }
  return total;
}

bool ChainsFit(ShahdSession* s, const StepPlan* plans, const int* r0, int nchain) {
  for (int c = 0; c < nchain; c++) {
    const StepPlan& p = plans[c];
    if (p.M < 1 || r0[c] < 0 || r0[c] + p.M > s->rows_cap ||
        ((p.finish || (p.head && p.am_val == nullptr)) && r0[c] + p.M > s->max_seqs)) {
      SetError("internal: step of rows [%d, %d) exceeds the session's row buffers", r0[c], r0[c] + p.M);
      return false;
    }
  }
  return true;
}

// Run a step (or concurrent chains of steps) through a cached CUDA graph. The first use of a shape runs
// eagerly (lazy host-side setup such as kernel attributes and TMA descriptors stays out of capture), the
// second captures it, every later one replays it. In measurement mode the graph also holds an event node
// on each side of every kernel, and each replay is waited for and its kernel times added up.
int RunStep(ShahdSession* s, const StepPlan* plans, const int* r0, int nchain, int kind, int reps = 1) {
  if (!ChainsFit(s, plans, r0, nchain)) return SHAHD_EINVAL;
  // `reps` consecutive steps in one graph: every input of a decode step (tokens, positions, outputs) lives
  // on the device, so back-to-back steps need no host update in between
  auto enqueue = [&]() {
    int total = 0;
    StepPlan pl[kMaxChains];
    for (int c = 0; c < nchain; c++) pl[c] = plans[c];
    for (int j = 0; j < reps; j++) {
      s->cur_rep = j;
      total += EnqueueChains(s, pl, r0, nchain);
      for (int c = 0; c < nchain; c++) pl[c].embed_ready = EmbedsNext(pl[c]);  // the finish kernel embedded the next input
    }
    s->cur_rep = 0;
    return total;
  };
  s->chains_hint = nchain;
  if (s->prof) SHAHD_TRY(HarvestEager(s));  // eager records before the step, so graph records stay apart
  const StepPlan& p = plans[0];
  GraphKey key{(reps * 16 + kind) * 16 + nchain, p.M, p.slot, p.tok, p.poff, p.prompt, p.out_ids, p.out_ld,
               g_umma_min_rows * 4 + (int)g_use_pdl * 2 + (int)s->prof,
               p.sampling.temperature > 0 ? p.sampling.temperature : 0.0,
               p.sampling.temperature > 0 ? p.sampling.top_p : 1.0, p.sampling.temperature > 0 ? p.sampling.top_k : 0,
               p.logits, (int)p.head + 2 * (int)p.embed_ready, p.plan_i0, p.plan_n, p.plan_qblocks};
  auto it = s->graphs.find(key);
  if (it == s->graphs.end()) {
    enqueue();
    SHAHD_TRY(CheckLaunch("step"));
    s->graphs.emplace(key, StepGraph{nullptr, 0, {}});
    if (s->prof) SHAHD_TRY(HarvestEager(s));
    return SHAHD_OK;
  }
  if (it->second.exec == nullptr) {
    cudaGraph_t g = nullptr;
    SHAHD_CUDA_TRY(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
    const long long saved = s->launches;
    s->capturing = true;
    const int n = enqueue();
    s->capturing = false;
    s->launches = saved;
    std::string where;
    const cudaError_t le = TakeLaunchError(&where);
    it->second.recs.swap(s->prof_recs);
    s->prof_recs.clear();
    cudaError_t e = cudaStreamEndCapture(s->stream, &g);
    if (le != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      SetError("step capture: %s failed: %s", where.c_str(), cudaGetErrorString(le));
      return SHAHD_ECUDA;
    }
    if (e != cudaSuccess) {
      SetError("step capture failed: %s", cudaGetErrorString(e));
      return SHAHD_ECUDA;
    }
    e = cudaGraphInstantiate(&it->second.exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      it->second.exec = nullptr;
      SetError("step graph instantiate failed: %s", cudaGetErrorString(e));
      return SHAHD_ECUDA;
    }
    it->second.launches = n;
  }
  SHAHD_CUDA_TRY(cudaGraphLaunch(it->second.exec, s->stream));
  s->launches += it->second.launches;
  if (s->prof) {
    SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
    SHAHD_TRY(Accumulate(s, it->second.recs, plans));
  }
  return SHAHD_OK;
}

int RunStep(ShahdSession* s, const StepPlan& p, int kind) {
  const int r0 = 0;
  return RunStep(s, &p, &r0, 1, kind);
}

// ---- KV page management (host mirror of the block table) ---------------------------------------

void ResetSlot(ShahdSession* s, int slot) {
  for (int b = 0; b < s->max_blocks; b++) {
    int& e = s->h_block_table[slot * s->max_blocks + b];
    if (e >= 0) {
      s->free_pages.push_back(e);
      e = -1;
    }
  }
  s->h_len[slot] = 0;
}

// Pages for positions [0, upto) of `slot`.
int EnsurePages(ShahdSession* s, int slot, int upto) {
  const int need = std::min(CeilDiv(upto, kPageTokens), s->max_blocks);
  for (int b = 0; b < need; b++) {
    int& e = s->h_block_table[slot * s->max_blocks + b];
    if (e < 0) {
      if (s->free_pages.empty()) {
        SetError("KV pool exhausted: no free page for slot %d position %d (kv_pages=%d)", slot, b * kPageTokens,
                 s->kv_pages);
        return SHAHD_ENOMEM;
      }
      e = s->free_pages.back();
      s->free_pages.pop_back();
    }
  }
  return SHAHD_OK;
}

// Block table and lengths to the device. The pinned mirror is only modified while the session stream is
// idle, so the asynchronous copy reads the values of this call.
int UploadTables(ShahdSession* s) {
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_block_table, s->h_block_table, sizeof(int) * (size_t)s->max_seqs * s->max_blocks,
                                 cudaMemcpyHostToDevice, s->stream));
  return SHAHD_OK;
}

int* Staging(ShahdSession* s, int row) { return s->h_pinned_rows + (size_t)row * s->max_seqs; }

int UploadLengths(ShahdSession* s) {
  int* h = Staging(s, kStagingLengths);  // not a prefill-plan row: that copy may still be pending
  std::copy(s->h_len.begin(), s->h_len.end(), h);
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_seq_len, h, sizeof(int) * s->max_seqs, cudaMemcpyHostToDevice, s->stream));
  return SHAHD_OK;
}

__global__ void GatherLastTokens(const int* prompt, const int* ends, int n, int* cur) {
  int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < n) cur[r] = prompt[ends[r] - 1];
}

// Window rebuild input: the last `keep` ids of prompt_r ++ out_r[0..gen) (CachedForward.ts:133-141).
__global__ void GatherWindow(const int* prompt, const int* pstart, const int* plen, const int* out, int out_ld,
                             const int* rows, int nrows, int gen, int keep, int* window) {
  int i = blockIdx.x;
  if (i >= nrows) return;
  int r = rows[i];
  int total = plen[r] + gen;
  int start = total - keep;
  for (int k = threadIdx.x; k < keep; k += blockDim.x) {
    int idx = start + k;
    window[(size_t)i * keep + k] = idx < plen[r] ? prompt[pstart[r] + idx] : out[(size_t)r * out_ld + (idx - plen[r])];
  }
}

__global__ void SetLengths(int* seq_len, const int* slots, int n, int value) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) seq_len[slots[i]] = value;
}

// Expands per-sequence prefill plans into rows: sequence i of [i0, i1) contributes rows
// (row_off[i] - row_off[i0]) + t for t < len[i], each with its slot, position t and gather offset.
__global__ void ExpandPrefillRows(const int* plan, int max_seqs, int i0, int i1, int* row_slot, int* row_pos,
                                  int* row_poff) {
  const int i = i0 + blockIdx.x;
  if (i >= i1) return;
  const int slot = plan[i], start = plan[max_seqs + i], len = plan[2 * max_seqs + i];
  const int off = plan[3 * max_seqs + i] - plan[3 * max_seqs + i0], base = plan[4 * max_seqs + i];
  for (int t = threadIdx.x; t < len; t += blockDim.x) {
    row_slot[off + t] = slot;
    row_pos[off + t] = base + t;     // the row's token is prompt[start + t] = prompt[poff + position]
    row_poff[off + t] = start - base;
  }
}

// PrefillCache (CachedForward.ts:100-110) for several slots at once: every prompt position of every
// sequence is one row of a batched blocks-only step (no LM head); QKV writes each row's K/V at its
// position before the attention of the same step reads positions 0..t of the row's slot, which is the
// causal mask of the reference's tensor forward. Sequences go in chunks of whole sequences of at most
// rows_cap rows. Slots must be reset with pages assigned; ids of sequence i are d_prompt[start_i + t].
// Outputs of a verify pass: a head over every appended row (logits and per-row greedy ids).
struct VerifyOut {
  float* logits;  // [rows, V]
  float* am_val;  // [rows, am_stride] argmax partials
  int* am_idx;
  int* ids;       // [rows]
};

__global__ void ArgmaxRowsKernel(const float* am_val, const int* am_idx, int nblk, int rows, int* ids) {
  const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int b = lane; b < nblk; b += 32) ArgmaxMerge(bv, bi, am_val[(size_t)r * nblk + b], am_idx[(size_t)r * nblk + b]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    ArgmaxMerge(bv, bi, ov, oi);
  }
  if (lane == 0) ids[r] = bi == 0x7fffffff ? 0 : bi;
}

// Appends slot i's tokens d_prompt[starts[i] + t], t < lens[i], at positions bases[i] + t (0 when bases is
// null: PrefillCache). With `vo` (a verify pass, one chunk only) the LM head also runs on every row.
int PrefillBatched(ShahdSession* s, const int* d_prompt, const std::vector<int>& slots, const std::vector<int>& starts,
                   const std::vector<int>& lens, const std::vector<int>* bases = nullptr,
                   const VerifyOut* vo = nullptr) {
  const int n = (int)slots.size(), R = s->max_seqs;
  int* h = Staging(s, 8);  // rows 8..12: slot, start, len, row offset, base position
  long long off = 0;
  for (int i = 0; i < n; i++) {
    h[i] = slots[i];
    h[R + i] = starts[i];
    h[2 * R + i] = lens[i];
    h[3 * R + i] = (int)off;
    h[4 * R + i] = bases ? (*bases)[i] : 0;
    off += lens[i];
  }
  if (off > 0) {
    SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_seq_plan, h, sizeof(int) * 5 * (size_t)R, cudaMemcpyHostToDevice, s->stream));
    for (int i0 = 0; i0 < n;) {
      int i1 = i0, rows = 0;
      long long attended = 0;
      while (i1 < n && rows + lens[i1] <= s->rows_cap) {
        const long long b = bases ? (*bases)[i1] : 0;
        rows += lens[i1];
        attended += (long long)lens[i1] * b + (long long)lens[i1] * (lens[i1] + 1) / 2;
        i1++;
      }
      if (i1 == i0 || (vo && i1 < n)) {  // a sequence longer than a chunk: rows_cap >= block_size rules this out
        SetError("PrefillCache: %lld tokens exceed the chunk of %d rows", vo ? off : (long long)lens[i0], s->rows_cap);
        return SHAHD_EINVAL;
      }
      if (rows > 0) {
        ExpandPrefillRows<<<i1 - i0, 128, 0, s->stream>>>(s->d_seq_plan, R, i0, i1, s->d_row_slot, s->d_row_pos,
                                                           s->d_row_poff);
        s->launches++;
        StepPlan p{rows, s->d_row_pos, false, s->d_row_slot, nullptr, s->d_row_poff, d_prompt, vo != nullptr,
                   vo ? vo->logits : nullptr, nullptr, nullptr, nullptr, 0, attended};
        int longest = 0;
        for (int i = i0; i < i1; i++) {
          longest = std::max(longest, lens[i]);
          const long long b = bases ? (*bases)[i] : 0;
          for (int qb = 0; qb < lens[i]; qb += kPfQ) p.kv_streamed += b + std::min(lens[i], qb + kPfQ);
        }
        p.seq_plan = s->d_seq_plan;
        p.plan_i0 = i0;
        p.plan_n = i1 - i0;
        p.plan_qblocks = CeilDiv(longest, kPfQ);
        if (vo) {
          p.am_val = vo->am_val;
          p.am_idx = vo->am_idx;
        }
        SHAHD_TRY(RunStep(s, p, 0));
        if (vo) {
          ArgmaxRowsKernel<<<CeilDiv(rows, 4), 128, 0, s->stream>>>(vo->am_val, vo->am_idx, HeadBlocks(s, rows), rows,
                                                                    vo->ids);
          s->launches++;
        }
      }
      i0 = i1;
    }
  }
  for (int i = 0; i < n; i++) s->h_len[slots[i]] = (bases ? (*bases)[i] : 0) + lens[i];
  SHAHD_TRY(UploadLengths(s));
  return CheckLaunch("prefill");
}

int ValidateSlots(ShahdSession* s, const int32_t* slots, int n, const char* op) {
  std::vector<char> seen(s->max_seqs, 0);
  for (int i = 0; i < n; i++) {
    if (slots[i] < 0 || slots[i] >= s->max_seqs) {
      SetError("%s: slot %d out of range [0,%d)", op, slots[i], s->max_seqs);
      return SHAHD_EINVAL;
    }
    if (seen[slots[i]]) {
      SetError("%s: slot %d listed twice", op, slots[i]);
      return SHAHD_EINVAL;
    }
    seen[slots[i]] = 1;
  }
  return SHAHD_OK;
}

int ValidateIds(ShahdSession* s, const int32_t* ids, size_t n, const char* op) {
  for (size_t i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= s->V) {
      SetError("%s: token id %d out of range [0,%d) — likely a tokenizer/vocab mismatch", op, ids[i], s->V);
      return SHAHD_EINVAL;
    }
  return SHAHD_OK;
}

int GrowPrompt(ShahdSession* s, size_t count) {
  if (count <= s->prompt_cap) return SHAHD_OK;
  size_t cap = std::max(count, s->prompt_cap * 2);
  int* p = nullptr;
  SHAHD_TRY(DevAlloc(s, &p, cap));
  s->d_prompt = p;
  s->prompt_cap = cap;
  return SHAHD_OK;
}

int GrowOut(ShahdSession* s, size_t count) {
  if (count <= s->out_cap) return SHAHD_OK;
  size_t cap = std::max(count, s->out_cap * 2);
  int* p = nullptr;
  SHAHD_TRY(DevAlloc(s, &p, cap));
  s->d_out = p;
  s->out_cap = cap;
  return SHAHD_OK;
}

// ---- persistent cluster decode loop: eligibility, shared-memory plan, launch ------------------------

using LoopKernelFn = void (*)(const LoopDesc);
constexpr size_t kLoopSmemBudget = 227 * 1024;  // dynamic shared memory of one CTA at most

LoopKernelFn LoopKernelFor(int d, int G) {
  const int mg = G <= 1 ? 1 : (G <= 2 ? 2 : 4);
  if (d == 64) return mg == 1 ? DecodeLoopKernel<64, 1> : (mg == 2 ? DecodeLoopKernel<64, 2> : DecodeLoopKernel<64, 4>);
  return mg == 1 ? DecodeLoopKernel<32, 1> : (mg == 2 ? DecodeLoopKernel<32, 2> : DecodeLoopKernel<32, 4>);
}

// Shared-memory plan of a launch whose clusters hold `rows` rows; returns the bytes (0: does not fit).
size_t LoopPlan(const ShahdSession* s, int rows, LoopDesc* D) {
  const int max_items = CeilDiv(rows * s->Hk, kLoopCS);
  const int nq = CeilDiv(CeilDiv(s->Nqkv, 128), kLoopCS), nu = CeilDiv(CeilDiv(s->Nup, 128), kLoopCS);
  const int gd = s->G * s->d;
  // the shape fields the per-CTA schedule depends on (CTA 0 holds the most tiles and attention items)
  D->E = s->E; D->Ep = s->Ep; D->H = s->H; D->Hk = s->Hk; D->d = s->d; D->G = s->G; D->F = s->F; D->Fp = s->Fp;
  D->V = s->V; D->L = s->L; D->HDp = s->HDp; D->Nqkv = s->Nqkv; D->Nup = s->Nup; D->mlp_kind = s->cfg.mlp_kind;
  const size_t budget = kLoopSmemBudget - 1024;  // the kernel aligns its base to 1024 bytes
  for (int boxes = kLoopMaxStageBoxes; boxes >= 1; boxes /= 2) {
    D->stage_boxes = boxes;
    const LoopSched S0 = MakeSched(*D, 0, max_items);
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) {
      off = (off + align - 1) / align * align;
      const size_t at = off;
      off += bytes;
      return (int)at;
    };
    // everything after the ring; the ring depth is chosen last
    D->off_xb = take((size_t)(s->Ep / 64) * kLoopOpBlock, 1024);
    D->off_ctxb = take((size_t)CeilDiv(gd, 64) * kLoopOpBlock, 1024);
    D->off_actb = take((size_t)nu * LoopActKb(s->cfg.mlp_kind) * kLoopOpBlock, 1024);
    D->off_xf = take((size_t)kLoopRows * s->E * 4, 16);
    D->off_qkv = take((size_t)nq * kLoopRows * 128 * 4, 16);
    D->off_opart = take((size_t)max_items * s->E * 4, 16);
    D->off_dpart = take((size_t)s->E * kLoopRows * 4, 16);
    D->off_xs = take((size_t)kLoopRows * (s->E / kLoopCS) * 4, 16);
    D->off_att = take((size_t)std::max(kLoopWarps, max_items) * (2 * s->G + gd) * 4, 16);
    D->off_sq = take((size_t)max_items * gd * 4, 16);
    D->off_rope = take((size_t)2 * kLoopRows * (s->d / 2) * 4, 16);
    D->off_sched = take((size_t)std::max(1, S0.per_step) * sizeof(LoopStage), 16);
    D->off_misc = take(sizeof(LoopMisc), 16);
    const size_t tail = off;
    const size_t stage_bytes = (size_t)boxes * kLoopBoxBytes;
    if (tail + 2 * stage_bytes > budget) continue;  // at least two stages in flight
    const int stages = (int)std::min<size_t>(kLoopMaxStages, (budget - tail) / stage_bytes);
    const int ring = stages * (int)stage_bytes;
    D->off_xb += ring; D->off_ctxb += ring; D->off_actb += ring; D->off_xf += ring; D->off_qkv += ring;
    D->off_opart += ring; D->off_dpart += ring; D->off_xs += ring; D->off_att += ring; D->off_sq += ring;
    D->off_rope += ring; D->off_sched += ring; D->off_misc += ring;
    D->stages = stages;
    D->max_items = max_items;
    return ring + tail + 1024;
  }
  return 0;
}

// The decode loop runs greedy decode steps of models whose shapes fit its fixed work split: head_dim 32 or
// 64, at most four query heads per kv head, kv heads dividing the cluster, E a multiple of 64 up to 512,
// at most four QKV / MLP-up tiles of 128 features per CTA. One-time set-up per session: tensor maps of
// every weight (box 64 x 128), the per-layer constants, kernel attributes and the resident-cluster count.
bool LoopSetup(ShahdSession* s) {
  if (s->loop_state >= 0) return s->loop_state == 1;
  s->loop_state = 0;
  if (!(s->d == 32 || s->d == 64) || s->G > 4 || kLoopCS % s->Hk != 0) return false;
  if (s->E % 64 != 0 || s->E > 512 || s->Ep != s->E || s->L > kLoopMaxLayers) return false;
  if (CeilDiv(CeilDiv(s->Nqkv, 128), kLoopCS) > kLoopMaxTiles || CeilDiv(CeilDiv(s->Nup, 128), kLoopCS) > kLoopMaxTiles ||
      CeilDiv(s->E, 128) > kLoopMaxTiles)
    return false;
  static thread_local LoopDesc D;
  D = LoopDesc{};
  if (LoopPlan(s, kLoopRows, &D) == 0) return false;
  // every plan (any rows per cluster: fewer rows leave room for a deeper weight ring) fits the budget
  const size_t smem = kLoopSmemBudget;
  const LoopKernelFn fn = LoopKernelFor(s->d, s->G);
  if (!EnsureKernelAttrs((const void*)fn, (int)smem, true)) {
    TakeLaunchError(nullptr);  // not an error of the caller's run: the per-kernel path takes over
    return false;
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(kLoopCS * 8);
  lc.blockDim = dim3(kLoopThreads);
  lc.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kLoopCS;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  int nclusters = 0;
  if (cudaOccupancyMaxActiveClusters(&nclusters, (void*)fn, &lc) != cudaSuccess || nclusters < 1) {
    cudaGetLastError();
    return false;
  }
  std::vector<CUtensorMap> wm(4 * s->L + 1);
  for (int l = 0; l < s->L; l++) {
    const Layer& Ly = s->layers[l];
    if (!MakeTmaBf16(Ly.w_qkv, s->Nqkv, s->Ep, s->Ep, 128, &wm[4 * l]) ||
        !MakeTmaBf16(Ly.w_o, s->E, s->HDp, s->HDp, 128, &wm[4 * l + 1]) ||
        !MakeTmaBf16(Ly.w_up, s->Nup, s->Ep, s->Ep, 128, &wm[4 * l + 2]) ||
        !MakeTmaBf16(Ly.w_down, s->E, s->Fp, s->Fp, 128, &wm[4 * l + 3]))
      return false;
  }
  if (!MakeTmaBf16(s->w_head, s->V, s->Ep, s->Ep, 128, &wm[4 * s->L])) return false;
  std::vector<LoopLayer> ly(s->L);
  for (int l = 0; l < s->L; l++) {
    const Layer& Ly = s->layers[l];
    ly[l] = LoopLayer{Ly.qkv_c1, Ly.qkv_c2, Ly.up_c1, Ly.up_c2, Ly.b_fc, Ly.b_proj};
  }
  if (DevAlloc(s, &s->d_loop_layers, ly.size()) != SHAHD_OK) return false;
  if (cudaMemcpy(s->d_loop_layers, ly.data(), sizeof(LoopLayer) * ly.size(), cudaMemcpyHostToDevice) != cudaSuccess)
    return false;
  s->loop_wmaps = wm;
  s->loop_max_clusters = nclusters;
  s->loop_state = 1;
  return true;
}

// Rows per cluster for n rows: spread them over the clusters that are resident at once (more clusters only
// queue behind the first wave), at most kLoopRows each.
int LoopRows(const ShahdSession* s, int n) {
  const int clusters = std::max(1, std::min(s->loop_max_clusters, n));
  return std::min(kLoopRows, CeilDiv(n, clusters));
}

// Algorithmic bytes of `steps` decode steps of n rows whose cached lengths before the first step are `len`:
// every weight matrix once per step, each row's cached K/V rows read and its new K/V row written.
double LoopBytes(const ShahdSession* s, const std::vector<int>& len, int n, int steps) {
  const double w = 2.0 * ((double)s->L * ((double)s->Nqkv * s->E + (double)s->E * s->H * s->d + (double)s->Nup * s->E +
                                          (double)s->E * s->F) + (double)s->V * s->E);
  const double per_pos = (double)s->L * s->Hk * 2 * s->d * 2;
  double kv = 0;
  for (int i = 0; i < n; i++)
    for (int k = 0; k < steps; k++) kv += per_pos * (len[i] + k + 1) + per_pos;
  return w * steps + kv;
}

// Launches the decode loop for `steps` greedy steps of rows 0..n-1 (slots d_slot, inputs d_tok); the ids of
// step k land in out[:, gen0 + k]. logits (nullable, device [n, steps, V]) records every step's logits.
int LaunchLoop(ShahdSession* s, int n, int steps, int* d_out, int out_ld, int gen0, float* logits) {
  const int rows = LoopRows(s, n);
  static thread_local LoopDesc D;  // 8 KB of tensor maps: kept off the stack
  D = LoopDesc{};
  const size_t smem = LoopPlan(s, rows, &D);
  D.M = n; D.E = s->E; D.Ep = s->Ep; D.H = s->H; D.Hk = s->Hk; D.d = s->d; D.G = s->G; D.F = s->F; D.Fp = s->Fp;
  D.V = s->V; D.L = s->L; D.HDp = s->HDp; D.Nqkv = s->Nqkv; D.Nup = s->Nup;
  D.norm = s->cfg.norm_kind == 1 ? kNormRms : kNormLayer;
  D.mlp_kind = s->cfg.mlp_kind;
  D.rows = rows;
  D.steps = steps;
  D.gen0 = gen0;
  D.out_ld = out_ld;
  D.eps = (float)s->cfg.layer_norm_eps;
  D.scale = (float)(1.0 / std::sqrt((double)s->d));
  D.slot = s->d_slot; D.tok = s->d_tok; D.seq_len = s->d_seq_len; D.out_ids = d_out; D.gen_count = s->d_gen_count;
  D.logits = logits;
  D.wte = s->wte; D.wpe = s->wpe; D.rope_cos = s->rope_cos; D.rope_sin = s->rope_sin;
  D.head_bias = s->head_bias; D.head_c1 = s->head_c1; D.head_c2 = s->head_c2;
  D.kv = KvView{s->kv_pool, s->d_block_table, s->max_blocks, s->Hk, s->d, s->page_elems};
  D.layers = s->d_loop_layers;
  std::copy(s->loop_wmaps.begin(), s->loop_wmaps.end(), D.wmaps);
  D.trace = nullptr;
  D.trace_steps = 0;
  if (std::getenv("SHAHD_LOOP_TRACE") != nullptr) {
    D.trace_steps = std::min(steps, 8);
    const size_t nt = (size_t)D.trace_steps * (s->L + 1) * kLoopMarks;
    if (s->loop_trace_cap < nt) {
      SHAHD_TRY(DevAlloc(s, &s->d_loop_trace, nt));
      s->loop_trace_cap = nt;
    }
    SHAHD_CUDA_TRY(cudaMemsetAsync(s->d_loop_trace, 0, nt * 8, s->stream));
    D.trace = s->d_loop_trace;
  }
  const LoopKernelFn fn = LoopKernelFor(s->d, s->G);
  const int clusters = CeilDiv(n, rows);
  cudaError_t err = cudaSuccess;
  std::vector<int> len(n);
  for (int i = 0; i < n; i++) len[i] = s->h_len[i];
  Timed(s, s->stream, kProfLoop, LoopBytes(s, len, n, steps), [&] {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(clusters * kLoopCS);
    lc.blockDim = dim3(kLoopThreads);
    lc.dynamicSmemBytes = smem;
    lc.stream = s->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = kLoopCS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    err = cudaLaunchKernelEx(&lc, fn, D);
  });
  if (err != cudaSuccess) {
    SetError("decode loop launch failed: %s", cudaGetErrorString(err));
    return SHAHD_ECUDA;
  }
  if (D.trace) {  // diagnostics: per-phase timestamps of the first steps, appended to SHAHD_LOOP_TRACE
    const size_t nt = (size_t)D.trace_steps * (s->L + 1) * kLoopMarks;
    std::vector<unsigned long long> h(nt);
    SHAHD_CUDA_TRY(cudaMemcpyAsync(h.data(), D.trace, nt * 8, cudaMemcpyDeviceToHost, s->stream));
    SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
    if (FILE* f = std::fopen(std::getenv("SHAHD_LOOP_TRACE"), "a")) {
      std::fprintf(f, "# rows %d rows_per_cluster %d clusters %d stages %d steps %d layers %d\n", n, rows,
                   CeilDiv(n, rows), D.stages, steps, s->L);
      for (size_t i = 0; i < nt; i += kLoopMarks) {
        std::fprintf(f, "%zu %zu", i / kLoopMarks / (s->L + 1), (i / kLoopMarks) % (s->L + 1));
        for (int k = 0; k < kLoopMarks; k++) std::fprintf(f, " %llu", h[i + k]);
        std::fprintf(f, "\n");
      }
      std::fclose(f);
    }
  }
  return SHAHD_OK;
}

// Whether a generate call runs its decode steps in the persistent loop.
bool UseLoop(ShahdSession* s, int n, const ShahdSampling* o) {
  return g_persistent_step && !(o && o->temperature > 0) && n >= 1 && n <= s->max_seqs && LoopSetup(s);
}

// Core of shahd_generate / shahd_generate_device on the session stream. d_prompt_packed holds the packed
// prompts on the device; offs their host offsets. Output ids land in d_out [n, max_new].
int GenerateCore(ShahdSession* s, const int* d_prompt_packed, const std::vector<int>& offs, int n, int max_new,
                 const ShahdSampling* o, int* d_out, float* d_logits = nullptr) {
  const bool sample = o && o->temperature > 0;
  const int C = s->C;
  // CachedDecoder constructor: Context = prompt.slice(-BlockSize); prefill all but its last id.
  std::vector<int> plen(n), pstart(n), full_len(n), slots(n);
  for (int i = 0; i < n; i++) {
    full_len[i] = offs[i + 1] - offs[i];
    const int ctx = std::min(full_len[i], C);
    pstart[i] = offs[i + 1] - ctx;
    plen[i] = ctx - 1;
    slots[i] = i;
  }
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));  // pinned staging and tables are rewritten below
  for (int i = 0; i < n; i++) ResetSlot(s, i);
  // Pages for the whole run up front: positions reach min(plen + max_new, C).
  for (int i = 0; i < n; i++) SHAHD_TRY(EnsurePages(s, i, std::min(plen[i] + max_new, C)));
  SHAHD_TRY(UploadTables(s));

  int *h_slot = Staging(s, 2), *h_ends = Staging(s, 3), *h_starts = Staging(s, 4), *h_full = Staging(s, 5);
  for (int i = 0; i < n; i++) {
    h_slot[i] = i;
    h_ends[i] = offs[i + 1];
    h_starts[i] = offs[i];
    h_full[i] = full_len[i];
  }
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_slot, h_slot, sizeof(int) * n, cudaMemcpyHostToDevice, s->stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_ends, h_ends, sizeof(int) * n, cudaMemcpyHostToDevice, s->stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_starts, h_starts, sizeof(int) * n, cudaMemcpyHostToDevice, s->stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_full_len, h_full, sizeof(int) * n, cudaMemcpyHostToDevice, s->stream));
  SHAHD_CUDA_TRY(cudaMemsetAsync(s->d_gen_count, 0, sizeof(int) * n, s->stream));

  SHAHD_TRY(PrefillBatched(s, d_prompt_packed, slots, pstart, plen));
  GatherLastTokens<<<CeilDiv(n, 128), 128, 0, s->stream>>>(d_prompt_packed, s->d_ends, n, s->d_tok);
  s->launches++;
  // the decode loop: step k consumes the last context id (k = 0) or the id sampled at k-1. Greedy runs of
  // supported shapes go through the persistent cluster loop; otherwise rows are split into chains of
  // per-kernel steps (independent sequences on their own streams).
  const bool loop = UseLoop(s, n, o);
  if (d_logits && !loop) {
    SetError("logits recording needs a greedy run of a model the decode loop supports");
    return SHAHD_EINVAL;
  }
  const int nchain = DecodeChains(n);
  StepPlan plans[kMaxChains];
  int r0[kMaxChains];
  for (int c = 0; c < nchain; c++) {
    r0[c] = c * n / nchain;
    const int rows = (c + 1) * n / nchain - r0[c];
    plans[c] = StepPlan{rows, nullptr, true, s->d_slot + r0[c], s->d_tok + r0[c], nullptr, nullptr, true, nullptr,
                        nullptr, s->d_tok + r0[c], d_out + (size_t)r0[c] * max_new, max_new, 0};
    if (sample) {
      plans[c].logits = s->logits + (size_t)r0[c] * s->V;  // the sampler reads the head's logits
      plans[c].sampling = *o;
    }
  }
  for (int k = 0; k < max_new; k++) {
    // rows whose window is full rebuild it from their last C-1 ids first (CachedForward.ts:135-141)
    std::vector<int> slide;
    for (int i = 0; i < n; i++)
      if (s->h_len[i] >= C) slide.push_back(i);
    if (!slide.empty()) {
      const int keep = C - 1;
      const int ns = (int)slide.size();
      SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));  // staging rows 6, 7 and 8-11 are rewritten
      int* h_rows = Staging(s, 6);
      std::vector<int> wstart(ns), wlen(ns, keep);
      for (int i = 0; i < ns; i++) {
        h_rows[i] = slide[i];
        wstart[i] = i * keep;  // gather offsets into the window buffer
      }
      SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_rows, h_rows, sizeof(int) * ns, cudaMemcpyHostToDevice, s->stream));
      GatherWindow<<<ns, 128, 0, s->stream>>>(d_prompt_packed, s->d_starts, s->d_full_len, d_out, max_new, s->d_rows,
                                              ns, k - 1, keep, s->d_window);
      s->launches++;
      SHAHD_TRY(PrefillBatched(s, s->d_window, slide, wstart, wlen));
      for (int c = 0; c < nchain; c++) plans[c].embed_ready = false;  // the rebuild reused the activation rows
    }
    for (int c = 0; c < nchain; c++) {
      plans[c].attended = 0;
      for (int i = r0[c]; i < r0[c] + plans[c].M; i++) plans[c].attended += s->h_len[i] + 1;
    }
    int maxlen = 0;
    for (int i = 0; i < n; i++) maxlen = std::max(maxlen, s->h_len[i]);
    if (loop) {  // every step until the next window rebuild (or the end) in one persistent launch
      const int steps = std::max(1, std::min(max_new - k, C - maxlen));
      SHAHD_TRY(LaunchLoop(s, n, steps, d_out, max_new, k, d_logits));
      for (int i = 0; i < n; i++) s->h_len[i] += steps;
      k += steps - 1;
      continue;
    }
    // consecutive steps that need no window rebuild go into one graph
    const int reps = std::max(1, std::min({kStepsPerGraph, max_new - k, C - maxlen}));
    SHAHD_TRY(RunStep(s, plans, r0, nchain, 1, reps));
    for (int c = 0; c < nchain; c++) plans[c].embed_ready = EmbedsNext(plans[c]);  // next input embedded
    for (int i = 0; i < n; i++) s->h_len[i] += reps;
    k += reps - 1;
  }
  return CheckLaunch("generate");
}

// Join a caller stream: our stream waits for work already queued on `caller`, and at exit the caller
// waits for ours.
void JoinIn(ShahdSession* s, cudaStream_t caller) {
  if (caller == s->stream) return;
  cudaEventRecord(s->join_in, caller);
  cudaStreamWaitEvent(s->stream, s->join_in, 0);
}
void JoinOut(ShahdSession* s, cudaStream_t caller) {
  if (caller == s->stream) return;
  cudaEventRecord(s->join_out, s->stream);
  cudaStreamWaitEvent(caller, s->join_out, 0);
}

}  // namespace
}  // namespace shahd

using namespace shahd;

// ================================================================================================
// C ABI
// ================================================================================================

extern "C" int64_t shahd_param_count(const ShahdModelCfg* cfg) {
  ClearError();
  ParamLayout lay;
  if (!cfg || BuildParamLayout(*cfg, &lay) != SHAHD_OK) return -1;
  return lay.total;
}

extern "C" int shahd_session_create(const ShahdModelCfg* cfg, const void* params, int32_t params_f64,
                                    int64_t params_count, const ShahdSessionOpts* opts, ShahdSession** out) {
  ClearError();
  if (!cfg || !params || !opts || !out) {
    SetError("shahd_session_create: null argument");
    return SHAHD_EINVAL;
  }
  *out = nullptr;
  ParamLayout lay;
  if (BuildParamLayout(*cfg, &lay) != SHAHD_OK) return SHAHD_EINVAL;
  if (params_count != lay.total) {
    SetError("shahd_session_create: params hold %lld values but the model needs %lld", (long long)params_count,
             (long long)lay.total);
    return SHAHD_EINVAL;
  }
  if (opts->max_seqs < 1) {
    SetError("shahd_session_create: max_seqs must be >= 1, got %d", opts->max_seqs);
    return SHAHD_EINVAL;
  }
  const int d = cfg->embed_dim / cfg->num_heads;
  if (d % 2 != 0 || d > kMaxHeadDimGeneric) {
    SetError("shahd_session_create: head dim %d must be even and <= %d", d, kMaxHeadDimGeneric);
    return SHAHD_EINVAL;
  }
  if (cfg->num_heads / cfg->kv_heads > kMaxGroup) {
    SetError("shahd_session_create: query group %d exceeds %d", cfg->num_heads / cfg->kv_heads, kMaxGroup);
    return SHAHD_EINVAL;
  }
  if ((size_t)16 * RoundUp(std::max(cfg->embed_dim, cfg->mlp_hidden), 8) * 4 > 224 * 1024) {
    SetError("shahd_session_create: EmbedDim/MlpHidden above 3584 are not supported by the row kernels");
    return SHAHD_EINVAL;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || opts->device < 0 || opts->device >= ndev) {
    SetError("shahd_session_create: CUDA device %d not available", opts->device);
    return SHAHD_ENODEV;
  }
  cudaDeviceProp prop;
  SHAHD_CUDA_TRY(cudaGetDeviceProperties(&prop, opts->device));
  if (prop.major != 10) {
    SetError("shahd_session_create: device %d is sm_%d%d, this build runs on sm_100", opts->device, prop.major, prop.minor);
    return SHAHD_ENODEV;
  }
  SHAHD_CUDA_TRY(cudaSetDevice(opts->device));

  ShahdSession* s = new ShahdSession();
  s->cfg = *cfg;
  s->E = cfg->embed_dim; s->L = cfg->num_layers; s->H = cfg->num_heads; s->Hk = cfg->kv_heads; s->d = d;
  s->F = cfg->mlp_hidden; s->C = cfg->block_size; s->V = cfg->vocab_size; s->G = s->H / s->Hk;
  s->Ep = RoundUp(s->E, 8); s->Fp = RoundUp(s->F, 8); s->HDp = RoundUp(s->H * d, 8);
  s->Nqkv = (s->H + 2 * s->Hk) * d;
  s->Nup = cfg->mlp_kind == 0 ? s->F : 2 * s->F;
  s->device = opts->device;
  s->max_seqs = opts->max_seqs;
  s->rows_cap = std::max(s->max_seqs, std::max(kPrefillRows, s->C));
  cudaDeviceGetAttribute(&s->num_sms, cudaDevAttrMultiProcessorCount, opts->device);
  s->max_blocks = CeilDiv(s->C, kPageTokens);
  s->kv_pages = opts->kv_pages > 0 ? opts->kv_pages : s->max_seqs * s->max_blocks;
  s->page_elems = (size_t)s->L * s->Hk * 2 * kPageTokens * d;
  auto fail = [&](int rc) {
    shahd_session_destroy(s);
    return rc;
  };
  bool streams_ok = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) == cudaSuccess &&
                    cudaEventCreateWithFlags(&s->join_in, cudaEventDisableTiming) == cudaSuccess &&
                    cudaEventCreateWithFlags(&s->join_out, cudaEventDisableTiming) == cudaSuccess &&
                    cudaEventCreateWithFlags(&s->fork_ev, cudaEventDisableTiming) == cudaSuccess;
  for (int c = 0; c < kMaxChains - 1 && streams_ok; c++)
    streams_ok = cudaStreamCreateWithFlags(&s->side[c], cudaStreamNonBlocking) == cudaSuccess &&
                 cudaEventCreateWithFlags(&s->chain_ev[c], cudaEventDisableTiming) == cudaSuccess;
  if (!streams_ok) {
    SetError("cudaStreamCreate/cudaEventCreate failed");
    return fail(SHAHD_ECUDA);
  }

  // ---- weights: repack on the host, one copy each ----
  HostWeights hw;
  if (RepackWeights(*cfg, lay, params, params_f64 != 0, &hw) != SHAHD_OK) return fail(SHAHD_EINVAL);
  auto up_bf = [&](const std::vector<bf16>& v, bf16** dst) -> int {
    SHAHD_TRY(DevAlloc(s, dst, v.size()));
    SHAHD_CUDA_TRY(cudaMemcpy(*dst, v.data(), v.size() * sizeof(bf16), cudaMemcpyHostToDevice));
    return SHAHD_OK;
  };
  auto up_f = [&](const std::vector<float>& v, float** dst) -> int {
    if (v.empty()) {
      *dst = nullptr;
      return SHAHD_OK;
    }
    SHAHD_TRY(DevAlloc(s, dst, v.size()));
    SHAHD_CUDA_TRY(cudaMemcpy(*dst, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
    return SHAHD_OK;
  };
  int rc = SHAHD_OK;
  s->layers.resize(s->L);
  for (int l = 0; l < s->L && rc == SHAHD_OK; l++) {
    Layer& Ly = s->layers[l];
    const HostLayer& hl = hw.layers[l];
    rc = up_bf(hl.w_qkv, &Ly.w_qkv);
    if (rc == SHAHD_OK) rc = up_bf(hl.w_o, &Ly.w_o);
    if (rc == SHAHD_OK) rc = up_bf(hl.w_up, &Ly.w_up);
    if (rc == SHAHD_OK) rc = up_bf(hl.w_down, &Ly.w_down);
    if (rc == SHAHD_OK) rc = up_f(hl.qkv_c1, &Ly.qkv_c1);
    if (rc == SHAHD_OK) rc = up_f(hl.qkv_c2, &Ly.qkv_c2);
    if (rc == SHAHD_OK) rc = up_f(hl.up_c1, &Ly.up_c1);
    if (rc == SHAHD_OK) rc = up_f(hl.up_c2, &Ly.up_c2);
    if (rc == SHAHD_OK) rc = up_f(hl.b_fc, &Ly.b_fc);
    if (rc == SHAHD_OK) rc = up_f(hl.b_proj, &Ly.b_proj);
  }
  if (rc == SHAHD_OK) rc = up_bf(hw.w_head, &s->w_head);
  if (rc == SHAHD_OK) rc = up_f(hw.head_bias, &s->head_bias);
  if (rc == SHAHD_OK) rc = up_f(hw.head_c1, &s->head_c1);
  if (rc == SHAHD_OK) rc = up_f(hw.head_c2, &s->head_c2);
  if (rc == SHAHD_OK) rc = up_f(hw.wte, &s->wte);
  if (rc == SHAHD_OK) rc = up_f(hw.wpe, &s->wpe);
  if (rc == SHAHD_OK) rc = up_f(hw.rope_cos, &s->rope_cos);
  if (rc == SHAHD_OK) rc = up_f(hw.rope_sin, &s->rope_sin);
  if (rc != SHAHD_OK) return fail(rc);

  // ---- KV pool + tables ----
  const int R = s->max_seqs;
  if ((rc = DevAlloc(s, &s->kv_pool, s->page_elems * (size_t)s->kv_pages)) != SHAHD_OK) return fail(rc);
  // positions a page has not been written at hold zeros: a masked key's probability is exactly zero, and the
  // tensor-core P.V must not meet a non-finite leftover there
  cudaMemset(s->kv_pool, 0, sizeof(bf16) * s->page_elems * (size_t)s->kv_pages);
  if (s->d == kFaD) {
    const long long rows = (long long)s->page_elems / s->d * s->kv_pages;
    s->kv_tmap_ok = rows < (1LL << 31) && MakeTmaBf16(s->kv_pool, (int)rows, s->d, s->d, kPageTokens, &s->kv_tmap);
  }
  if ((rc = DevAlloc(s, &s->d_block_table, (size_t)R * s->max_blocks)) != SHAHD_OK) return fail(rc);
  if ((rc = DevAlloc(s, &s->d_seq_len, (size_t)R)) != SHAHD_OK) return fail(rc);
  if (cudaMallocHost(&s->h_block_table, sizeof(int) * (size_t)R * s->max_blocks) != cudaSuccess ||
      cudaMallocHost(&s->h_pinned_rows, sizeof(int) * (size_t)R * kStagingRows) != cudaSuccess) {
    SetError("cudaMallocHost failed");
    return fail(SHAHD_ENOMEM);
  }
  std::fill(s->h_block_table, s->h_block_table + (size_t)R * s->max_blocks, -1);
  s->free_pages.resize(s->kv_pages);
  for (int i = 0; i < s->kv_pages; i++) s->free_pages[i] = s->kv_pages - 1 - i;
  s->h_len.assign(R, 0);

  // ---- per-row scratch ----
  s->am_stride = std::max(CeilDiv(s->V, kSimtCols), UmmaGridN(s->V));  // argmax partials per decode row
  const size_t hd = (size_t)s->H * d;
  const size_t RC = (size_t)s->rows_cap;  // activation rows (decode rows or one prefill chunk)
  if ((rc = DevAlloc(s, &s->x, RC * s->E)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->xb, RC * s->Ep)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->q, RC * hd)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->ctx, RC * hd)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->ctxb, RC * s->HDp)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->act, RC * s->F)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->actb, RC * s->Fp)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->logits, (size_t)R * s->V)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->am_val, (size_t)R * s->am_stride)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->am_idx, (size_t)R * s->am_stride)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->part_o, (size_t)R * s->H * s->max_blocks * d)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->part_m, (size_t)R * s->H * s->max_blocks)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->part_l, (size_t)R * s->H * s->max_blocks)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->attn_counter, (size_t)R * s->Hk)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->row_stats, 2 * RC)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_slot, (size_t)R)) != SHAHD_OK || (rc = DevAlloc(s, &s->d_tok, (size_t)R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_pos, RC)) != SHAHD_OK ||  // one position per row, prefill rows included
      (rc = DevAlloc(s, &s->d_next, (size_t)R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_gen_count, (size_t)R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_ends, (size_t)R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_starts, (size_t)R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_full_len, (size_t)R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_rows, (size_t)R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_rng, (size_t)R)) != SHAHD_OK || (rc = DevAlloc(s, &s->d_sampled, (size_t)R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_seq_plan, (size_t)5 * R)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_row_slot, (size_t)s->rows_cap)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_row_pos, (size_t)s->rows_cap)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_row_poff, (size_t)s->rows_cap)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->d_window, (size_t)R * s->C)) != SHAHD_OK)
    return fail(rc);
  s->split_ws_floats = std::max(UmmaKSplitFloats(s->E, s->HDp), UmmaKSplitFloats(s->E, s->Fp));
  s->split_cnt_len = CeilDiv(s->E, 16);
  if ((rc = DevAlloc(s, &s->split_ws, s->split_ws_floats * kMaxChains)) != SHAHD_OK ||
      (rc = DevAlloc(s, &s->split_cnt, (size_t)s->split_cnt_len * kMaxChains)) != SHAHD_OK)
    return fail(rc);
  cudaMemset(s->split_cnt, 0, sizeof(int) * (size_t)s->split_cnt_len * kMaxChains);
  // bf16 operand rows are read over their padded width: padding columns must stay zero
  cudaMemset(s->xb, 0, sizeof(bf16) * RC * s->Ep);
  cudaMemset(s->ctxb, 0, sizeof(bf16) * RC * s->HDp);
  cudaMemset(s->actb, 0, sizeof(bf16) * RC * s->Fp);
  // per-device kernel attributes (a process may hold sessions on several devices)
  TakeLaunchError(nullptr);
  if (!EnsureKernelAttrs((const void*)AttnDecodeKernel<32>, AttnSmemBytes(32)) ||
      !EnsureKernelAttrs((const void*)AttnDecodeKernel<64>, AttnSmemBytes(64)) ||
      !EnsureKernelAttrs((const void*)AttnDecodeKernel<128>, AttnSmemBytes(128)) ||
      !EnsureKernelAttrs((const void*)PrefillAttnKernel<32>, PrefillAttnSmem(32)) ||
      !EnsureKernelAttrs((const void*)PrefillAttnKernel<64>, PrefillAttnSmem(64)) ||
      !EnsureKernelAttrs((const void*)PrefillAttnKernel<128>, PrefillAttnSmem(128)) ||
      !EnsureKernelAttrs((const void*)PrefillAttnUmmaKernel, kFaSmemLaunch) || !EnsureAttnPagesAttrs<32>() ||
      !EnsureAttnPagesAttrs<64>() || !EnsureAttnPagesAttrs<128>()) {
    TakeLaunchError(nullptr);
    SetError("shahd_session_create: kernel attributes could not be set on device %d", s->device);
    return fail(SHAHD_ECUDA);
  }
  cudaMemset(s->attn_counter, 0, sizeof(int) * (size_t)R * s->Hk);
  s->ab_ok = AttnBlockFits(s->d, s->G, s->Hk, s->E, s->Ep) && EnsureAttnBlockAttrs(s->d, s->G, s->Ep);
  TakeLaunchError(nullptr);
  cudaMemset(s->d_seq_len, 0, sizeof(int) * R);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    SetError("shahd_session_create: device error during setup");
    return fail(SHAHD_ECUDA);
  }
  *out = s;
  return SHAHD_OK;
}

extern "C" int shahd_session_destroy(ShahdSession* s) {
  if (!s) return SHAHD_OK;
  cudaSetDevice(s->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  for (auto& kv : s->graphs)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  for (cudaEvent_t e : s->ev_pool) cudaEventDestroy(e);
  for (cudaEvent_t e : s->graph_events) cudaEventDestroy(e);
  for (void* p : s->allocs) {
    auto it = s->alloc_bytes.find(p);
    ForgetTmaRange(p, static_cast<char*>(p) + (it != s->alloc_bytes.end() ? it->second : 1));  // maps into it go stale
    cudaFree(p);
  }
  if (s->h_block_table) cudaFreeHost(s->h_block_table);
  if (s->h_pinned_rows) cudaFreeHost(s->h_pinned_rows);
  for (int c = 0; c < kMaxChains - 1; c++) {
    if (s->side[c]) cudaStreamSynchronize(s->side[c]), cudaStreamDestroy(s->side[c]);
    if (s->chain_ev[c]) cudaEventDestroy(s->chain_ev[c]);
  }
  if (s->fork_ev) cudaEventDestroy(s->fork_ev);
  if (s->join_in) cudaEventDestroy(s->join_in);
  if (s->join_out) cudaEventDestroy(s->join_out);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
  return SHAHD_OK;
}

extern "C" int shahd_reset(ShahdSession* s, const int32_t* slots, int32_t n) {
  ClearError();
  if (!s || (n > 0 && !slots) || n < 0) {
    SetError("shahd_reset: bad arguments");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_TRY(ValidateSlots(s, slots, n, "shahd_reset"));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  for (int i = 0; i < n; i++) ResetSlot(s, slots[i]);
  SHAHD_TRY(UploadTables(s));
  SHAHD_TRY(UploadLengths(s));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  return SHAHD_OK;
}

extern "C" int32_t shahd_seq_length(ShahdSession* s, int32_t slot) {
  ClearError();
  if (!s || slot < 0 || slot >= s->max_seqs) {
    SetError("shahd_seq_length: bad slot");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  return s->h_len[slot];
}

extern "C" int shahd_prefill(ShahdSession* s, const int32_t* slots, const int32_t* ids, const int32_t* offsets, int32_t n) {
  ClearError();
  if (!s || n < 0 || (n > 0 && (!slots || !offsets))) {
    SetError("shahd_prefill: bad arguments");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_TRY(ValidateSlots(s, slots, n, "shahd_prefill"));
  size_t total = 0;
  for (int i = 0; i < n; i++) {
    const int len = offsets[i + 1] - offsets[i];
    if (offsets[i] < 0 || len < 0) {
      SetError("shahd_prefill: offsets must be non-decreasing from 0");
      return SHAHD_EINVAL;
    }
    if (len > s->C) {
      SetError("PrefillCache: %d tokens exceed the cache capacity %d", len, s->C);
      return SHAHD_EINVAL;
    }
    total = offsets[i + 1];
  }
  if (total > 0 && !ids) {
    SetError("shahd_prefill: ids is null");
    return SHAHD_EINVAL;
  }
  SHAHD_TRY(ValidateIds(s, ids, total, "PrefillCache"));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  for (int i = 0; i < n; i++) ResetSlot(s, slots[i]);
  std::vector<int> sl(slots, slots + n), starts(n), lens(n);
  for (int i = 0; i < n; i++) {
    starts[i] = offsets[i];
    lens[i] = offsets[i + 1] - offsets[i];
    SHAHD_TRY(EnsurePages(s, sl[i], lens[i]));
  }
  SHAHD_TRY(UploadTables(s));
  if (total > 0) {
    SHAHD_TRY(GrowPrompt(s, total));
    SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_prompt, ids, sizeof(int) * total, cudaMemcpyHostToDevice, s->stream));
  }
  SHAHD_TRY(PrefillBatched(s, s->d_prompt, sl, starts, lens));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  return SHAHD_OK;
}

extern "C" int shahd_step(ShahdSession* s, const int32_t* slots, const int32_t* tokens, int32_t n, float* logits,
                          int32_t* next_ids) {
  ClearError();
  if (!s || n < 1 || !slots || !tokens) {
    SetError("shahd_step: bad arguments");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  if (n > s->max_seqs) {
    SetError("shahd_step: %d rows exceed max_seqs %d", n, s->max_seqs);
    return SHAHD_EINVAL;
  }
  SHAHD_TRY(ValidateSlots(s, slots, n, "shahd_step"));
  SHAHD_TRY(ValidateIds(s, tokens, n, "CachedForwardStep"));
  for (int i = 0; i < n; i++)
    if (s->h_len[slots[i]] >= s->C) {
      SetError("CachedForwardStep: position %d is outside the %d-token window — rebuild the cache", s->h_len[slots[i]],
               s->C);
      return SHAHD_EINVAL;
    }
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  for (int i = 0; i < n; i++) SHAHD_TRY(EnsurePages(s, slots[i], s->h_len[slots[i]] + 1));
  SHAHD_TRY(UploadTables(s));
  int *h_sl = Staging(s, 0), *h_tk = Staging(s, 1);
  std::copy(slots, slots + n, h_sl);
  std::copy(tokens, tokens + n, h_tk);
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_slot, h_sl, sizeof(int) * n, cudaMemcpyHostToDevice, s->stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_tok, h_tk, sizeof(int) * n, cudaMemcpyHostToDevice, s->stream));
  StepPlan p{n, nullptr, true, s->d_slot, s->d_tok, nullptr, nullptr, true, logits ? s->logits : nullptr, s->d_next, nullptr,
             nullptr, 0, 0};
  for (int i = 0; i < n; i++) p.attended += s->h_len[slots[i]] + 1;
  if (EnqueueStep(s, p, s->stream) < 0) return SHAHD_EINVAL;
  SHAHD_TRY(CheckLaunch("shahd_step"));
  for (int i = 0; i < n; i++) s->h_len[slots[i]] += 1;
  if (logits)
    SHAHD_CUDA_TRY(cudaMemcpyAsync(logits, s->logits, sizeof(float) * (size_t)n * s->V, cudaMemcpyDeviceToHost, s->stream));
  if (next_ids) SHAHD_CUDA_TRY(cudaMemcpyAsync(next_ids, s->d_next, sizeof(int) * n, cudaMemcpyDeviceToHost, s->stream));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  return SHAHD_OK;
}

static int ValidateGenerate(ShahdSession* s, const int32_t* offsets, int32_t n, int32_t max_new) {
  if (n < 1 || n > s->max_seqs) {
    SetError("shahd_generate: %d sequences, session holds %d", n, s->max_seqs);
    return SHAHD_EINVAL;
  }
  if (max_new < 0) {
    SetError("shahd_generate: max_new must be >= 0");
    return SHAHD_EINVAL;
  }
  if (offsets[0] != 0) {
    SetError("shahd_generate: offsets[0] must be 0");
    return SHAHD_EINVAL;
  }
  for (int i = 0; i < n; i++)
    if (offsets[i + 1] - offsets[i] < 1) {
      SetError("CachedGenerate: empty prompt — nothing to condition on (sequence %d)", i);
      return SHAHD_EINVAL;
    }
  return SHAHD_OK;
}

// Seeded sampling needs one SeededRng state per sequence and knobs the sampler can honour.
int ValidateSampling(ShahdSession* s, const ShahdSampling* o, const void* rng, const char* op) {
  if (!o || !(o->temperature > 0)) return SHAHD_OK;  // greedy (Temperature <= 0) draws nothing
  if (!std::isfinite(o->temperature) || std::isnan(o->top_p)) {
    SetError("%s: sampling temperature must be finite and top_p a number", op);
    return SHAHD_EINVAL;
  }
  if (!rng) {
    SetError("%s: temperature > 0 needs one SeededRng state per sequence (rng_states is null)", op);
    return SHAHD_EINVAL;
  }
  if (s->V > (1 << 22)) {
    SetError("%s: seeded sampling supports vocabularies up to %d ids, got %d", op, 1 << 22, s->V);
    return SHAHD_EINVAL;
  }
  return SHAHD_OK;
}

extern "C" int shahd_generate(ShahdSession* s, const int32_t* prompts, const int32_t* offsets, int32_t n, int32_t max_new,
                              const ShahdSampling* opts, uint32_t* rng_states, int32_t* out_ids) {
  ClearError();
  if (!s || !prompts || !offsets || (max_new > 0 && !out_ids)) {
    SetError("shahd_generate: null argument");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_TRY(ValidateGenerate(s, offsets, n, max_new));
  const size_t total = offsets[n];
  SHAHD_TRY(ValidateIds(s, prompts, total, "CachedGenerate"));
  SHAHD_TRY(ValidateSampling(s, opts, rng_states, "shahd_generate"));
  if (max_new == 0) return SHAHD_OK;  // CachedGenerate returns the prompt untouched, no prefill
  const bool sample = opts && opts->temperature > 0;
  std::vector<int> offs(offsets, offsets + n + 1);
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  SHAHD_TRY(GrowPrompt(s, total));
  SHAHD_TRY(GrowOut(s, (size_t)n * max_new));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_prompt, prompts, sizeof(int) * total, cudaMemcpyHostToDevice, s->stream));
  uint32_t* h_rng = reinterpret_cast<uint32_t*>(Staging(s, 0));  // staging row 0: free during a generate
  if (sample) {
    std::memcpy(h_rng, rng_states, sizeof(uint32_t) * n);
    SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_rng, h_rng, sizeof(uint32_t) * n, cudaMemcpyHostToDevice, s->stream));
  }
  SHAHD_TRY(GenerateCore(s, s->d_prompt, offs, n, max_new, opts, s->d_out));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(out_ids, s->d_out, sizeof(int) * (size_t)n * max_new, cudaMemcpyDeviceToHost, s->stream));
  if (sample)
    SHAHD_CUDA_TRY(cudaMemcpyAsync(h_rng, s->d_rng, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost, s->stream));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  if (sample) std::memcpy(rng_states, h_rng, sizeof(uint32_t) * n);  // states advanced by one draw per token
  return SHAHD_OK;
}

extern "C" int shahd_generate_device(ShahdSession* s, const int32_t* d_prompts, const int32_t* host_offsets, int32_t n,
                                     int32_t max_new, const ShahdSampling* opts, uint32_t* d_rng_states, int32_t* d_out_ids,
                                     void* stream) {
  ClearError();
  if (!s || !d_prompts || !host_offsets || (max_new > 0 && !d_out_ids)) {
    SetError("shahd_generate_device: null argument");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_TRY(ValidateGenerate(s, host_offsets, n, max_new));
  SHAHD_TRY(ValidateSampling(s, opts, d_rng_states, "shahd_generate_device"));
  if (max_new == 0) return SHAHD_OK;
  const bool sample = opts && opts->temperature > 0;
  std::vector<int> offs(host_offsets, host_offsets + n + 1);
  cudaStream_t caller = stream ? static_cast<cudaStream_t>(stream) : s->stream;
  JoinIn(s, caller);
  if (sample)
    SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_rng, d_rng_states, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice, s->stream));
  int rc = GenerateCore(s, d_prompts, offs, n, max_new, opts, d_out_ids);
  if (rc == SHAHD_OK && sample) {
    const cudaError_t e =
        cudaMemcpyAsync(d_rng_states, s->d_rng, sizeof(uint32_t) * n, cudaMemcpyDeviceToDevice, s->stream);
    if (e != cudaSuccess) {
      SetError("shahd_generate_device: copying the RNG states back failed: %s", cudaGetErrorString(e));
      rc = SHAHD_ECUDA;
    }
  }
  JoinOut(s, caller);
  return rc;
}

extern "C" int shahd_generate_logits(ShahdSession* s, const int32_t* prompts, const int32_t* offsets, int32_t n,
                                     int32_t max_new, int32_t* out_ids, float* logits) {
  ClearError();
  if (!s || !prompts || !offsets || (max_new > 0 && (!out_ids || !logits))) {
    SetError("shahd_generate_logits: null argument");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_TRY(ValidateGenerate(s, offsets, n, max_new));
  const size_t total = offsets[n];
  SHAHD_TRY(ValidateIds(s, prompts, total, "CachedGenerate"));
  if (max_new == 0) return SHAHD_OK;
  if (!UseLoop(s, n, nullptr)) {
    SetError("shahd_generate_logits: needs the persistent decode loop (enabled, and a model it supports)");
    return SHAHD_EINVAL;
  }
  std::vector<int> offs(offsets, offsets + n + 1);
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  SHAHD_TRY(GrowPrompt(s, total));
  SHAHD_TRY(GrowOut(s, (size_t)n * max_new));
  const size_t nl = (size_t)n * max_new * s->V;
  if (nl > s->loop_logits_cap) {
    if (s->d_loop_logits) {
      cudaFree(s->d_loop_logits);
      s->allocs.erase(std::find(s->allocs.begin(), s->allocs.end(), (void*)s->d_loop_logits));
      s->alloc_bytes.erase((void*)s->d_loop_logits);
      s->d_loop_logits = nullptr;
      s->loop_logits_cap = 0;
    }
    SHAHD_TRY(DevAlloc(s, &s->d_loop_logits, nl));
    s->loop_logits_cap = nl;
  }
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_prompt, prompts, sizeof(int) * total, cudaMemcpyHostToDevice, s->stream));
  SHAHD_TRY(GenerateCore(s, s->d_prompt, offs, n, max_new, nullptr, s->d_out, s->d_loop_logits));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(out_ids, s->d_out, sizeof(int) * (size_t)n * max_new, cudaMemcpyDeviceToHost, s->stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(logits, s->d_loop_logits, sizeof(float) * nl, cudaMemcpyDeviceToHost, s->stream));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  return SHAHD_OK;
}

extern "C" int shahd_sync(ShahdSession* s) {
  ClearError();
  if (!s) return SHAHD_EINVAL;
  cudaSetDevice(s->device);
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  SHAHD_CUDA_TRY(cudaDeviceSynchronize());
  return SHAHD_OK;
}

extern "C" int32_t shahd_step_launches(ShahdSession* s, int32_t n) {
  if (!s) return -1;
  // embed + per layer (QKV, attention, O, up, down | fused attention block, up, down) + head + finish
  return 1 + (UsesFusedBlock(s, n, 0) ? 3 : 5) * s->L + 2;
}

extern "C" int shahd_profile(ShahdSession* s, int32_t enable) {
  ClearError();
  if (!s) return SHAHD_EINVAL;
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_CUDA_TRY(cudaDeviceSynchronize());
  s->prof = enable != 0;
  s->prof_recs.clear();
  s->ev_used = 0;
  for (int k = 0; k < kProfKinds; k++) {
    s->prof_ms[k] = s->prof_bytes[k] = 0;
    s->prof_n[k] = 0;
  }
  return SHAHD_OK;
}

extern "C" int shahd_profile_read(ShahdSession* s, int32_t kind, double* total_ms, int64_t* launches, double* bytes) {
  ClearError();
  if (!s || kind < 0 || kind >= kProfKinds || !total_ms || !launches || !bytes) {
    SetError("shahd_profile_read: bad arguments");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_CUDA_TRY(cudaDeviceSynchronize());
  SHAHD_TRY(HarvestEager(s));
  const double ms = s->prof_ms[kind], b = s->prof_bytes[kind];
  const int64_t n = s->prof_n[kind];
  *total_ms = ms;
  *launches = n;
  *bytes = b;
  return SHAHD_OK;
}

extern "C" int64_t shahd_kernel_launches(ShahdSession* s) { return s ? (int64_t)s->launches : -1; }

extern "C" int shahd_verify(ShahdSession* s, const int32_t* slots, const int32_t* tokens, const int32_t* offsets,
                            int32_t n, float* logits, int32_t* next_ids) {
  ClearError();
  if (!s || n < 1 || !slots || !tokens || !offsets || !next_ids) {
    SetError("shahd_verify: bad arguments");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_TRY(ValidateSlots(s, slots, n, "shahd_verify"));
  if (offsets[0] != 0) {
    SetError("shahd_verify: offsets must start at 0");
    return SHAHD_EINVAL;
  }
  std::vector<int> sl(slots, slots + n), starts(n), lens(n), bases(n);
  for (int i = 0; i < n; i++) {
    lens[i] = offsets[i + 1] - offsets[i];
    starts[i] = offsets[i];
    bases[i] = s->h_len[slots[i]];
    if (lens[i] < 1) {
      SetError("shahd_verify: sequence %d has no tokens to verify", i);
      return SHAHD_EINVAL;
    }
    if (bases[i] + lens[i] > s->C) {
      SetError("shahd_verify: slot %d would reach position %d, outside the %d-token window", slots[i],
               bases[i] + lens[i] - 1, s->C);
      return SHAHD_EINVAL;
    }
  }
  const int total = offsets[n];
  if (total > s->rows_cap) {
    SetError("shahd_verify: %d rows exceed the %d rows of one pass", total, s->rows_cap);
    return SHAHD_EINVAL;
  }
  SHAHD_TRY(ValidateIds(s, tokens, total, "shahd_verify"));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  for (int i = 0; i < n; i++) SHAHD_TRY(EnsurePages(s, sl[i], bases[i] + lens[i]));
  SHAHD_TRY(UploadTables(s));
  if (total > s->vrows_cap) {
    const int cap = std::max(total, 2 * s->vrows_cap);
    SHAHD_TRY(DevAlloc(s, &s->d_vlogits, (size_t)cap * s->V));
    SHAHD_TRY(DevAlloc(s, &s->d_vam_val, (size_t)cap * s->am_stride));
    SHAHD_TRY(DevAlloc(s, &s->d_vam_idx, (size_t)cap * s->am_stride));
    SHAHD_TRY(DevAlloc(s, &s->d_vids, (size_t)cap));
    s->vrows_cap = cap;
  }
  SHAHD_TRY(GrowPrompt(s, total));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(s->d_prompt, tokens, sizeof(int) * total, cudaMemcpyHostToDevice, s->stream));
  const VerifyOut vo{s->d_vlogits, s->d_vam_val, s->d_vam_idx, s->d_vids};
  SHAHD_TRY(PrefillBatched(s, s->d_prompt, sl, starts, lens, &bases, &vo));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(next_ids, s->d_vids, sizeof(int) * total, cudaMemcpyDeviceToHost, s->stream));
  if (logits)
    SHAHD_CUDA_TRY(
        cudaMemcpyAsync(logits, s->d_vlogits, sizeof(float) * (size_t)total * s->V, cudaMemcpyDeviceToHost, s->stream));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  return SHAHD_OK;
}

extern "C" int shahd_truncate(ShahdSession* s, const int32_t* slots, const int32_t* lengths, int32_t n) {
  ClearError();
  if (!s || n < 0 || (n > 0 && (!slots || !lengths))) {
    SetError("shahd_truncate: bad arguments");
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(s->mu);
  cudaSetDevice(s->device);
  SHAHD_TRY(ValidateSlots(s, slots, n, "shahd_truncate"));
  for (int i = 0; i < n; i++)
    if (lengths[i] < 0 || lengths[i] > s->h_len[slots[i]]) {
      SetError("shahd_truncate: slot %d holds %d positions, cannot keep %d", slots[i], s->h_len[slots[i]], lengths[i]);
      return SHAHD_EINVAL;
    }
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  for (int i = 0; i < n; i++) s->h_len[slots[i]] = lengths[i];
  SHAHD_TRY(UploadLengths(s));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(s->stream));
  return SHAHD_OK;
}

extern "C" int shahd_sample_logits(const float* logits, int32_t rows, int32_t vocab, const ShahdSampling* opts,
                                   uint32_t* rng_states, int32_t* out_ids) {
  const char* op = "shahd_sample_logits";
  ClearError();
  if (!logits || !out_ids || rows < 1 || vocab < 1) {
    SetError("%s: need logits and out_ids and rows, vocab >= 1 (got rows=%d vocab=%d)", op, rows, vocab);
    return SHAHD_EINVAL;
  }
  const bool sample = opts && opts->temperature > 0;
  if (sample) {
    if (!std::isfinite(opts->temperature) || std::isnan(opts->top_p) || !rng_states) {
      SetError("%s: temperature > 0 needs a finite temperature, a numeric top_p and rng_states", op);
      return SHAHD_EINVAL;
    }
    if (vocab > (1 << 22)) {
      SetError("%s: seeded sampling supports vocabularies up to %d ids, got %d", op, 1 << 22, vocab);
      return SHAHD_EINVAL;
    }
  }
  if (!DeviceOk()) {
    SetError("%s: no usable sm_100 device", op);
    return SHAHD_ENODEV;
  }
  int dev = 0;
  SHAHD_CUDA_TRY(cudaGetDevice(&dev));
  Workspace& w = WorkspaceFor(dev);
  std::lock_guard<std::mutex> g(w.mu);
  // [rows, vocab] f32 logits | rows rng states | rows ids | rows slots, each 256-byte aligned
  const auto align256 = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t nl = align256((size_t)rows * vocab * 4), nr = align256((size_t)rows * 4);
  const size_t need = nl + 3 * nr;
  if (w.cap < need) {
    if (w.buf) cudaFree(w.buf);
    w.buf = nullptr;
    w.cap = 0;
    SHAHD_CUDA_TRY(cudaMalloc(&w.buf, need));
    w.cap = need;
  }
  if (!w.stream) SHAHD_CUDA_TRY(cudaStreamCreateWithFlags(&w.stream, cudaStreamNonBlocking));
  uint8_t* base = static_cast<uint8_t*>(w.buf);
  float* d_logits = reinterpret_cast<float*>(base);
  uint32_t* d_rng = reinterpret_cast<uint32_t*>(base + nl);
  int* d_ids = reinterpret_cast<int*>(base + nl + nr);
  int* d_slot = reinterpret_cast<int*>(base + nl + 2 * nr);
  std::vector<int> slots(rows);
  std::iota(slots.begin(), slots.end(), 0);
  SHAHD_CUDA_TRY(cudaMemcpyAsync(d_logits, logits, (size_t)rows * vocab * 4, cudaMemcpyHostToDevice, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(d_slot, slots.data(), (size_t)rows * 4, cudaMemcpyHostToDevice, w.stream));
  if (sample) SHAHD_CUDA_TRY(cudaMemcpyAsync(d_rng, rng_states, (size_t)rows * 4, cudaMemcpyHostToDevice, w.stream));
  const SampleArgs sa{d_logits, vocab, d_slot, d_rng, sample ? (float)opts->temperature : 0.f, sample ? opts->top_k : 0,
                      sample ? opts->top_p : 1.0, d_ids};
  SampleKernel<<<rows, kSampleThreads, 0, w.stream>>>(sa);
  SHAHD_CUDA_TRY(cudaGetLastError());
  SHAHD_CUDA_TRY(cudaMemcpyAsync(out_ids, d_ids, (size_t)rows * 4, cudaMemcpyDeviceToHost, w.stream));
  if (sample) SHAHD_CUDA_TRY(cudaMemcpyAsync(rng_states, d_rng, (size_t)rows * 4, cudaMemcpyDeviceToHost, w.stream));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(w.stream));
  return SHAHD_OK;
}

extern "C" const char* shahd_last_error(void) { return GetError(); }

extern "C" int shahd_speculative_round(const float* target_logits, const float* draft_logits, const int32_t* proposals,
                                       const int32_t* g, const int32_t* budget, int32_t n, int32_t gamma,
                                       int32_t vocab, const ShahdSampling* opts, uint32_t* rng_states,
                                       int32_t* out_ids, int32_t* out_count, int32_t* accepted) {
  const char* op = "shahd_speculative_round";
  ClearError();
  if (!target_logits || !draft_logits || !proposals || !g || !budget || !opts || !rng_states || !out_ids ||
      !out_count || !accepted || n < 1 || gamma < 1 || vocab < 1) {
    SetError("%s: null buffer or n, gamma, vocab < 1 (n=%d gamma=%d vocab=%d)", op, n, gamma, vocab);
    return SHAHD_EINVAL;
  }
  if (!(opts->temperature > 0) || !std::isfinite(opts->temperature) || std::isnan(opts->top_p)) {
    SetError("%s: SpeculativeSample needs a finite temperature > 0 and a numeric top_p (greedy speculative "
             "decoding verifies argmax ids instead)", op);
    return SHAHD_EINVAL;
  }
  if (vocab > (1 << 22)) {
    SetError("%s: seeded sampling supports vocabularies up to %d ids, got %d", op, 1 << 22, vocab);
    return SHAHD_EINVAL;
  }
  for (int i = 0; i < n; i++) {
    if (g[i] < 0 || g[i] > gamma || budget[i] < 1) {
      SetError("%s: sequence %d has g=%d (0..%d) and budget=%d (>= 1)", op, i, g[i], gamma, budget[i]);
      return SHAHD_EINVAL;
    }
    for (int k = 0; k < g[i]; k++)
      if (proposals[(size_t)i * gamma + k] < 0 || proposals[(size_t)i * gamma + k] >= vocab) {
        SetError("%s: proposal %d of sequence %d is %d, outside [0,%d)", op, k, i, proposals[(size_t)i * gamma + k], vocab);
        return SHAHD_EINVAL;
      }
  }
  if (!DeviceOk()) {
    SetError("%s: no usable sm_100 device", op);
    return SHAHD_ENODEV;
  }
  int dev = 0;
  SHAHD_CUDA_TRY(cudaGetDevice(&dev));
  Workspace& w = WorkspaceFor(dev);
  std::lock_guard<std::mutex> lk(w.mu);
  const auto a256 = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t nt = (size_t)n * (gamma + 1) * vocab, nd = (size_t)n * gamma * vocab;
  const size_t bt = a256(nt * 4), bd = a256(nd * 4), bp = a256((size_t)n * gamma * 4), bn = a256((size_t)n * 4),
               bo = a256((size_t)n * (gamma + 1) * 4);
  const size_t need = bt + bd + bp + 3 * bn + bo + 2 * bn;
  if (w.cap < need) {
    if (w.buf) cudaFree(w.buf);
    w.buf = nullptr;
    w.cap = 0;
    SHAHD_CUDA_TRY(cudaMalloc(&w.buf, need));
    w.cap = need;
  }
  if (!w.stream) SHAHD_CUDA_TRY(cudaStreamCreateWithFlags(&w.stream, cudaStreamNonBlocking));
  uint8_t* b = static_cast<uint8_t*>(w.buf);
  float* d_t = reinterpret_cast<float*>(b);
  float* d_d = reinterpret_cast<float*>(b + bt);
  int* d_p = reinterpret_cast<int*>(b + bt + bd);
  int* d_g = reinterpret_cast<int*>(b + bt + bd + bp);
  int* d_b = reinterpret_cast<int*>(b + bt + bd + bp + bn);
  uint32_t* d_rng = reinterpret_cast<uint32_t*>(b + bt + bd + bp + 2 * bn);
  int* d_out = reinterpret_cast<int*>(b + bt + bd + bp + 3 * bn);
  int* d_cnt = reinterpret_cast<int*>(b + bt + bd + bp + 3 * bn + bo);
  int* d_acc = reinterpret_cast<int*>(b + bt + bd + bp + 3 * bn + bo + bn);
  SHAHD_CUDA_TRY(cudaMemcpyAsync(d_t, target_logits, nt * 4, cudaMemcpyHostToDevice, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(d_d, draft_logits, nd * 4, cudaMemcpyHostToDevice, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(d_p, proposals, (size_t)n * gamma * 4, cudaMemcpyHostToDevice, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(d_g, g, (size_t)n * 4, cudaMemcpyHostToDevice, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(d_b, budget, (size_t)n * 4, cudaMemcpyHostToDevice, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(d_rng, rng_states, (size_t)n * 4, cudaMemcpyHostToDevice, w.stream));
  const SpecArgs sa{d_t, d_d, d_p, d_g, d_b, gamma, vocab, d_rng, (float)opts->temperature, opts->top_k, opts->top_p,
                    d_out, d_cnt, d_acc};
  SpecRoundKernel<<<n, kSampleThreads, 0, w.stream>>>(sa);
  SHAHD_CUDA_TRY(cudaGetLastError());
  SHAHD_CUDA_TRY(cudaMemcpyAsync(out_ids, d_out, (size_t)n * (gamma + 1) * 4, cudaMemcpyDeviceToHost, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(out_count, d_cnt, (size_t)n * 4, cudaMemcpyDeviceToHost, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(accepted, d_acc, (size_t)n * 4, cudaMemcpyDeviceToHost, w.stream));
  SHAHD_CUDA_TRY(cudaMemcpyAsync(rng_states, d_rng, (size_t)n * 4, cudaMemcpyDeviceToHost, w.stream));
  SHAHD_CUDA_TRY(cudaStreamSynchronize(w.stream));
  return SHAHD_OK;
}
