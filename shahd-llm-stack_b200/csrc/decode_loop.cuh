// Persistent cluster decode loop (sm_100a): every greedy decode step of a CachedGenerate run in ONE launch.
//
// Restates the decode loop of CachedGenerate (Brain/Sampling/CachedForward.ts:153-171) with the cached step
// AdvanceOneToken + HeadLogitsRow (CachedForward.ts:32-96, CachedRowMath.ts:14-137) and ArgmaxOf
// (Distribution.ts:19-30) for independent sequences. Rows never depend on one another, so each thread-block
// cluster owns a group of up to 16 rows for all steps of the run and no two clusters ever synchronize.
//
// Inside a cluster of kLoopCS CTAs (one per SM) every projection is split by output features: a CTA
// multiplies 128-row tiles of the weights (M = 128, read by TMA into a ring of 16 KB stages) by the cluster's
// activation rows (N = 16, bf16, 128-byte-swizzled K-major operand in shared memory) with tcgen05.mma into
// TMEM ("swap AB": the weights are the wide operand, the rows the narrow one). Everything a CTA needs from a
// peer is PULLED from the peer's shared memory (ld.shared::cluster) after a cluster barrier, because remote
// loads are an order of magnitude faster than remote stores. One layer is four cluster barriers:
//   P1  row statistics of x (every CTA, from its fp32 copy), bf16 operand, QKV tiles + RoPE; K/V rows of the
//       step's position stored into the paged cache, q kept for the attention CTAs          -> barrier
//   P2  attention of the CTA's (row, kv head) items over the cache (online softmax, fp32), then the output
//       projection restricted to the item's head group (a K slice of Wo): partial rows       -> barrier
//   P3  every CTA sums all partial O rows into its own copy of x (same order everywhere, so the copies are
//       bit-identical), norm statistics, MLP up tile(s) + gate, then the down projection restricted to the
//       CTA's own slice of the hidden activations (a K slice of W_down): partial rows        -> barrier
//   P4  the owner of each slice of E/kLoopCS features sums the down partials of every CTA + residual -> barrier
//   next P1 (or the head) gathers the owners' slices back into every CTA's x.
// After the last layer every CTA runs its tiles of the LM head, keeps a per-row argmax candidate, and after one
// more barrier every CTA merges all candidates (ArgmaxOf: first index of the strict max) and embeds the chosen
// ids as the next step's input (EmbeddingLookup, Embedding.ts:14-26). Four barriers per layer + one per step.
//
// The thread that issues the MMAs also issues the weight loads: it keeps the ring topped up at every phase
// boundary (the schedule of weight k-blocks of a CTA is static), so the next phases' weights stream in while
// the current phase runs; one thread owning both ends of the ring cannot deadlock. Every wait is bounded: a
// timeout records kDevErrLoopTimeout, marks the CTA aborted (all later work is skipped, every barrier is still
// reached), waits for the loads in flight and releases TMEM.
#pragma once

#include "common.cuh"
#include "decode_kernels.cuh"

namespace shahd {

constexpr int kDevErrLoopTimeout = 5;

constexpr int kLoopCS = 16;                   // CTAs per cluster (non-portable cluster size)
constexpr int kLoopRows = 16;                 // rows per cluster at most (the MMA's N)
constexpr int kLoopWarps = 8;
constexpr int kLoopThreads = 32 * kLoopWarps;
constexpr int kLoopBoxBytes = 128 * 64 * 2;    // one weight k-block: 128 rows x 64 bf16 (one TMA box)
constexpr int kLoopMaxStageBoxes = 4;          // boxes of one ring stage (one barrier, one expect_tx) at most
constexpr int kLoopOpBlock = kLoopRows * 128;  // one operand k-block: 16 rows x 64 bf16, swizzled
constexpr int kLoopTmemCols = 512;
constexpr int kTmQkv = 0, kTmO = 64, kTmUp = 128, kTmDown = 192, kTmHead = 256;
constexpr int kLoopMaxTiles = 4;   // QKV / up tiles of one CTA, M-tiles of E (64 TMEM columns each region)
constexpr int kLoopHeadChunk = 16; // head tiles per TMEM chunk (256 columns)
constexpr int kLoopMaxStages = 6;

struct LoopLayer {
  const float *qkv_c1, *qkv_c2, *up_c1, *up_c2, *b_fc, *b_proj;
};

constexpr int kLoopMaxLayers = 16;
constexpr int kLoopMaxMaps = 4 * kLoopMaxLayers + 1;

// Shapes, pointers, weight tensor maps and the shared-memory plan of one launch (host-computed, passed by
// value as a __grid_constant__ parameter: the TMA unit reads the descriptors from the parameter bank).
struct LoopDesc {
  CUtensorMap wmaps[kLoopMaxMaps];  // qkv, o, up, down of each layer, then the head; box 64 x 128
  int M, E, Ep, H, Hk, d, G, F, Fp, V, L, HDp, Nqkv, Nup;
  int norm, mlp_kind;
  int rows;    // rows per cluster
  int steps;   // decode steps of this launch
  int stages;       // weight ring depth
  int stage_boxes;  // weight boxes per ring stage (1, 2 or 4): a phase's boxes are grouped into stages of this
  int gen0, out_ld;
  float eps, scale;
  const int* slot;  // [M]
  int* tok;         // [M] input id of the next step: read at entry, written back at exit
  int* seq_len;     // [slots] cached length: read at entry, written back at exit
  int* out_ids;     // [M, out_ld]: column gen0 + s receives step s's id
  int* gen_count;   // [M] advanced by steps
  float* logits;    // nullable [M, steps, V]
  const float *wte, *wpe, *rope_cos, *rope_sin, *head_bias, *head_c1, *head_c2;
  KvView kv;
  const LoopLayer* layers;   // [L]
  // dynamic shared memory plan: byte offsets from the 1024-aligned base
  int off_xb, off_ctxb, off_actb, off_xf, off_qkv, off_opart, off_dpart, off_xs, off_att, off_sq, off_rope, off_misc;
  int off_sched;  // the CTA's ring stages of one step: [per_step] LoopStage
  int max_items;
  unsigned long long* trace;  // nullable: per-phase timestamps [trace_steps][L + 1][kLoopMarks] (diagnostics)
  int trace_steps;
};

// Host and device agree on the per-CTA work split through these helpers.
__host__ __device__ inline int LoopCount(int total, int rank) { return total > rank ? (total - rank + kLoopCS - 1) / kLoopCS : 0; }
__host__ __device__ inline int LoopActKb(int mlp_kind) { return mlp_kind == 0 ? 2 : 1; }  // act k-blocks per up tile

struct LoopSched {
  int nkE, nkG, nE128, akb;
  int nq, no, nu, nh;      // tiles / M-tiles per phase of this CTA
  int bq, bo, bu, bd, bh;  // weight blocks (boxes) per phase
  int per_layer, per_step; // ring stages per layer and per step: a phase's boxes in groups of stage_boxes
};

// One ring stage of a CTA's static schedule: up to four weight boxes (tensor map, x, y), built once per launch.
struct LoopStage {
  int nbox;
  int map[kLoopMaxStageBoxes], x[kLoopMaxStageBoxes], y[kLoopMaxStageBoxes];
  int pad[3];
};

__host__ __device__ inline LoopSched MakeSched(const LoopDesc& D, int c, int n_items) {
  LoopSched S;
  S.nkE = D.Ep / 64;
  S.nkG = CeilDiv(D.G * D.d, 64);
  S.nE128 = CeilDiv(D.E, 128);
  S.akb = LoopActKb(D.mlp_kind);
  S.nq = LoopCount(CeilDiv(D.Nqkv, 128), c);
  S.nu = LoopCount(CeilDiv(D.Nup, 128), c);
  S.nh = LoopCount(CeilDiv(D.V, 128), c);
  S.no = n_items > 0 ? S.nE128 : 0;
  S.bq = S.nq * S.nkE;
  S.bo = S.no * S.nkG;
  S.bu = S.nu * S.nkE;
  S.bd = S.nu > 0 ? S.nE128 * S.nu * S.akb : 0;
  S.bh = S.nh * S.nkE;
  const int g = D.stage_boxes;
  S.per_layer = CeilDiv(S.bq, g) + CeilDiv(S.bo, g) + CeilDiv(S.bu, g) + CeilDiv(S.bd, g);
  S.per_step = D.L * S.per_layer + CeilDiv(S.bh, g);
  return S;
}

// Byte offset of element (row r, column k) of a [16 x K] bf16 operand in 128-byte-swizzled K-major k-blocks.
__device__ __forceinline__ uint32_t OpOffset(int r, int k) {
  return (uint32_t)((k >> 6) * kLoopOpBlock) + Sw128Offset(r, (k & 63) >> 3) + (uint32_t)((k & 7) * 2);
}

__device__ __forceinline__ unsigned long long GlobalTimerNs() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool MbarTestWait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(SmemAddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint32_t ClusterRank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared-memory window of CTA `rank` of the cluster for a local shared address.
__device__ __forceinline__ uint32_t PeerAddr(const void* p, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(SmemAddr(p)), "r"(rank));
  return ra;
}
__device__ __forceinline__ float4 LdPeer4(uint32_t a) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float LdPeer(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ int LdPeerI(uint32_t a) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

// Cluster barrier after possibly divergent code: the warp reconverges first (the barrier is .aligned).
__device__ __forceinline__ void LoopBarrier() {
  __syncwarp();
  ClusterSync();
}

__device__ __forceinline__ void PrefetchBulkL2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Per-CTA bookkeeping shared by all threads (lives in shared memory).
struct LoopMisc {
  uint64_t full[kLoopMaxStages];
  uint64_t empty[kLoopMaxStages];
  uint64_t mma_bar;
  uint32_t tmem;
  volatile int abort;
  int issued;  // weight blocks issued (thread 0's counter, published for the exit drain)
  int pos[kLoopRows], slot[kLoopRows], tok[kLoopRows], page[kLoopRows];
  float is[kLoopRows], mu[kLoopRows];
  float cand_v[kLoopRows];
  int cand_i[kLoopRows];
  float wcv[4][kLoopRows];
  int wci[4][kLoopRows];
};

// Position in a CTA's static schedule of weight k-blocks, advanced by increments: the one thread that walks
// the schedule would otherwise spend about a microsecond per block on integer divisions.
struct SchedCursor {
  int l, ph, t, u, kb;  // layer (or L: the head), phase (0 qkv, 1 o, 2 up, 3 down, 4 head), tile, up tile, k-block
  int bi;               // box index within the phase
};

struct LoopCtx {
  const LoopDesc& D;
  LoopSched S;
  LoopMisc* m;
  uint8_t* ring;
  int c;         // cluster rank
  int g_item;    // kv head of this CTA's attention items
  int total;     // weight blocks of the whole launch
  int cons;      // blocks consumed (thread 0)
  int iss;       // blocks issued (thread 0)
  int cst;       // ring slot of block `cons`, and the parity of its fill
  uint32_t cpar;
  int ist;       // ring slot of block `iss`, and the parity of that slot's current use
  uint32_t ipar;
  SchedCursor cur;  // schedule walker (builds the stage table)
  const LoopStage* sched;  // [per_step] this CTA's ring stages of one step (shared memory)
  int sidx;                // index in `sched` of stage `iss`
  uint32_t mma_phase;
  unsigned long long wait_full_ns, wait_mma_ns;  // thread 0's time in weight-stage and MMA waits (tracing)
  int blocking_topups;
  unsigned long long issue_ns, topup_ns;  // thread 0's time inside IssuePhase and inside TopUp (tracing)
};

__device__ __forceinline__ int PhaseTiles(const LoopSched& S, int ph) {
  return ph == 0 ? S.nq : ph == 1 ? S.no : ph == 2 ? S.nu : ph == 3 ? (S.nu > 0 ? S.nE128 : 0) : S.nh;
}
__device__ __forceinline__ int PhaseKb(const LoopSched& S, int ph) {
  return ph == 0 || ph == 2 || ph == 4 ? S.nkE : ph == 1 ? S.nkG : S.akb;
}
// Moves to the first phase with blocks at or after the cursor's phase (wrapping from the head to layer 0).
__device__ __forceinline__ void SkipEmpty(const LoopSched& S, int L, SchedCursor& k) {
  for (int guard = 0; guard < 8 * (L + 1) && PhaseTiles(S, k.ph) == 0; guard++) {
    if (k.ph == 4) { k.ph = 0; k.l = 0; }
    else if (k.ph == 3) { k.l++; k.ph = k.l == L ? 4 : 0; }
    else k.ph++;
  }
}
__device__ __forceinline__ int PhaseBoxes(const LoopSched& S, int ph) {
  return ph == 0 ? S.bq : ph == 1 ? S.bo : ph == 2 ? S.bu : ph == 3 ? S.bd : S.bh;
}
__device__ __forceinline__ void Advance(const LoopSched& S, int L, SchedCursor& k) {
  k.bi++;
  if (++k.kb < PhaseKb(S, k.ph)) return;
  k.kb = 0;
  if (k.ph == 3 && ++k.u < S.nu) return;
  k.u = 0;
  if (++k.t < PhaseTiles(S, k.ph)) return;
  k.t = 0;
  k.bi = 0;
  if (k.ph == 4) { k.ph = 0; k.l = 0; }
  else if (k.ph == 3) { k.l++; k.ph = k.l == L ? 4 : 0; }
  else k.ph++;
  SkipEmpty(S, L, k);
}
__device__ __forceinline__ void CursorCoords(const LoopDesc& D, const LoopSched& S, int c, int g_item,
                                             const SchedCursor& k, int& map, int& x, int& y) {
  switch (k.ph) {
    case 0: map = 4 * k.l; x = k.kb * 64; y = (c + k.t * kLoopCS) * 128; break;
    case 1: map = 4 * k.l + 1; x = g_item * D.G * D.d + k.kb * 64; y = k.t * 128; break;
    case 2: map = 4 * k.l + 2; x = k.kb * 64; y = (c + k.t * kLoopCS) * 128; break;
    case 3: map = 4 * k.l + 3; x = (c + k.u * kLoopCS) * 64 * S.akb + k.kb * 64; y = k.t * 128; break;
    default: map = 4 * D.L; x = k.kb * 64; y = (c + k.t * kLoopCS) * 128; break;
  }
}

// Thread 0, once per launch: the CTA's ring stages of one step (every step repeats them), each the next
// boxes of the current phase, at most stage_boxes of them (IssuePhase groups the boxes the same way).
__device__ __forceinline__ void BuildStageTable(LoopCtx& X, LoopStage* table) {
  const LoopDesc& D = X.D;
  for (int i = 0; i < X.S.per_step; i++) {
    LoopStage st{};
    st.nbox = min(D.stage_boxes, PhaseBoxes(X.S, X.cur.ph) - X.cur.bi);
    for (int j = 0; j < st.nbox; j++) {
      CursorCoords(D, X.S, X.c, X.g_item, X.cur, st.map[j], st.x[j], st.y[j]);
      Advance(X.S, D.L, X.cur);
    }
    table[i] = st;
  }
}

// Thread 0: fill ring stages while slots are free; with block_for_next, waits (bounded) for the slot of the
// stage the consumer needs next.
__device__ __forceinline__ void TopUpBody(LoopCtx& X, bool block_for_next) {
  const LoopDesc& D = X.D;
  const uint32_t stage_bytes = (uint32_t)D.stage_boxes * kLoopBoxBytes;
  while (X.iss < X.total && X.iss < X.cons + D.stages && !X.m->abort) {
    if (X.iss >= D.stages) {  // the slot's previous use must have been released by its MMAs
      if (block_for_next && X.iss == X.cons) {
        X.blocking_topups++;
        if (!MbarWaitBounded(&X.m->empty[X.ist], X.ipar ^ 1u, kWaitLimit)) {
          atomicCAS(&g_shahd_device_error, 0, kDevErrLoopTimeout);
          X.m->abort = 1;
          return;
        }
      } else if (!MbarTestWait(&X.m->empty[X.ist], X.ipar ^ 1u)) {
        return;
      }
    }
    const LoopStage& st = X.sched[X.sidx];
    uint64_t* bar = &X.m->full[X.ist];
    uint8_t* dst = X.ring + (size_t)X.ist * stage_bytes;
    MbarArriveExpectTx(bar, (uint32_t)(st.nbox * kLoopBoxBytes));
    for (int j = 0; j < st.nbox; j++) TmaLoad2D(dst + j * kLoopBoxBytes, &D.wmaps[st.map[j]], bar, st.x[j], st.y[j]);
    X.iss++;
    if (++X.sidx == X.S.per_step) X.sidx = 0;
    if (++X.ist == D.stages) {
      X.ist = 0;
      X.ipar ^= 1u;
    }
  }
}
__device__ __forceinline__ void TopUp(LoopCtx& X, bool block_for_next) {
  const unsigned long long t0 = X.D.trace ? GlobalTimerNs() : 0;
  TopUpBody(X, block_for_next);
  if (X.D.trace) X.topup_ns += GlobalTimerNs() - t0;
}

// Thread 0: MMAs of the `nblk` boxes of a phase (or of a chunk of whole stages of it); box k accumulates into
// TMEM columns col0 + 16 * (k / per_tile) with the operand's k-block (k % per_tile) at op_base (2 KB apart).
// Boxes arrive in ring stages of up to stage_boxes; kvalid_last: valid K of the last k-block of a tile
// (64 = full). Commits mma_bar at the end.
__device__ __forceinline__ void IssuePhase(LoopCtx& X, int nblk, int per_tile, uint32_t col0, uint32_t op_base,
                                           int kvalid_last) {
  const unsigned long long t_issue = X.D.trace ? GlobalTimerNs() : 0;
  const uint32_t idesc = UmmaIdescBf16(128, 16);
  const uint64_t ring_desc = SmemDescSw128(SmemAddr(X.ring));
  const uint64_t op_desc = SmemDescSw128(op_base);
  int kin = 0;
  uint32_t dcol = X.m->tmem + col0;
  for (int done = 0; done < nblk && !X.m->abort;) {
    const int nbox = min(X.D.stage_boxes, nblk - done);
    if (X.iss <= X.cons) TopUp(X, true);
    if (X.m->abort) break;
    const unsigned long long tw = X.D.trace ? GlobalTimerNs() : 0;
    const bool ok = MbarWaitBounded(&X.m->full[X.cst], X.cpar, kWaitLimit);
    if (X.D.trace) X.wait_full_ns += GlobalTimerNs() - tw;
    if (!ok) {
      atomicCAS(&g_shahd_device_error, 0, kDevErrLoopTimeout);
      X.m->abort = 1;
      break;
    }
    TcgenFenceAfter();
    uint64_t ad = ring_desc + (uint64_t)(X.cst * ((X.D.stage_boxes * kLoopBoxBytes) >> 4));
    for (int j = 0; j < nbox; j++, ad += (uint64_t)(kLoopBoxBytes >> 4)) {
      const uint64_t bd = op_desc + (uint64_t)(kin * (kLoopOpBlock >> 4));
      const int kv = (kin == per_tile - 1) ? kvalid_last : 64;
      for (int kk = 0; kk < kv / 16; kk++)
        UmmaBf16(dcol, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, (kin > 0 || kk > 0) ? 1u : 0u);
      if (++kin == per_tile) {
        kin = 0;
        dcol += 16u;
      }
    }
    UmmaCommit(&X.m->empty[X.cst]);
    X.cons++;
    if (++X.cst == X.D.stages) {
      X.cst = 0;
      X.cpar ^= 1u;
    }
    done += nbox;
    TopUp(X, false);
  }
  UmmaCommit(&X.m->mma_bar);  // also completes (vacuously) when nothing was issued
  if (X.D.trace) X.issue_ns += GlobalTimerNs() - t_issue;
}

// All threads: wait for the phase's MMAs (bounded), then fence for TMEM reads.
__device__ __forceinline__ void WaitMma(LoopCtx& X) {
  const uint32_t ph = X.mma_phase & 1;
  X.mma_phase++;
  const unsigned long long tw = X.D.trace ? GlobalTimerNs() : 0;
  const bool ok = MbarWaitBounded(&X.m->mma_bar, ph, kWaitLimit);
  if (X.D.trace) X.wait_mma_ns += GlobalTimerNs() - tw;
  if (!ok) {
    atomicCAS(&g_shahd_device_error, 0, kDevErrLoopTimeout);
    X.m->abort = 1;
  }
  TcgenFenceAfter();
}

// Writes one row's norm statistics (NormRow, CachedRowMath.ts:25-56) from its warp-reduced sums.
__device__ __forceinline__ void RowStatsFromSums(const LoopDesc& D, LoopMisc* m, int r, float s1, float s2, int lane) {
  s1 = WarpSum(s1);
  s2 = WarpSum(s2);
  if (lane == 0) {
    if (D.norm == kNormRms) {
      m->mu[r] = 0.f;
      m->is[r] = 1.0f / sqrtf(s2 / D.E + D.eps);
    } else {
      const float mu = s1 / D.E;
      m->mu[r] = mu;
      m->is[r] = 1.0f / sqrtf(fmaxf(s2 / D.E - mu * mu, 0.f) + D.eps);
    }
  }
}

// Stores 8 consecutive features of row r: fp32 into x, bf16 into the swizzled operand, and adds them to the
// row's sums.
__device__ __forceinline__ void PutChunk(const LoopDesc& D, float* xf, uint8_t* op, int r, int f, const float4& a,
                                         const float4& b, float& s1, float& s2) {
  *reinterpret_cast<float4*>(xf + (size_t)r * D.E + f) = a;
  *reinterpret_cast<float4*>(xf + (size_t)r * D.E + f + 4) = b;
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int j = 0; j < 8; j++) {
    s1 += v[j];
    s2 += v[j] * v[j];
  }
  StoreNbf<8>(reinterpret_cast<bf16*>(op + OpOffset(r, f)), v);
}

constexpr int kLoopMaxChunks = 2;  // 8-feature chunks per lane and row (E <= 512)

// One pass per row pair (warp w owns rows w and w + 8): the rows' embedding Wte[id] (+ Wpe[pos])
// (Embedding.ts:14-26) into x, their norm statistics and the bf16 MMA operand of the first layer. Rows past
// `nrows` are zero.
__device__ __forceinline__ void EmbedRows(const LoopDesc& D, float* xf, uint8_t* op, LoopMisc* m, int nrows, int warp,
                                          int lane) {
  const int nc = D.E / 8;
  float4 v[2][kLoopMaxChunks][2];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int r = warp + 8 * h;
#pragma unroll
    for (int i = 0; i < kLoopMaxChunks; i++) {
      const int c8 = lane + 32 * i, f = 8 * c8;
      v[h][i][0] = v[h][i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c8 < nc && r < nrows) {
        const float4* te = reinterpret_cast<const float4*>(D.wte + (size_t)m->tok[r] * D.E + f);
        v[h][i][0] = __ldg(te);
        v[h][i][1] = __ldg(te + 1);
        if (D.wpe) {
          const float4* pe = reinterpret_cast<const float4*>(D.wpe + (size_t)m->pos[r] * D.E + f);
          const float4 p0 = __ldg(pe), p1 = __ldg(pe + 1);
          v[h][i][0] = make_float4(v[h][i][0].x + p0.x, v[h][i][0].y + p0.y, v[h][i][0].z + p0.z, v[h][i][0].w + p0.w);
          v[h][i][1] = make_float4(v[h][i][1].x + p1.x, v[h][i][1].y + p1.y, v[h][i][1].z + p1.z, v[h][i][1].w + p1.w);
        }
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int r = warp + 8 * h;
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < kLoopMaxChunks; i++) {
      const int c8 = lane + 32 * i;
      if (c8 < nc) PutChunk(D, xf, op, r, 8 * c8, v[h][i][0], v[h][i][1], s1, s2);
    }
    RowStatsFromSums(D, m, r, s1, s2, lane);
  }
}

// The start of a layer (and of the head), in the same shape: x rows gathered from their owners' slices of
// E / CS features (each owner summed the down-projection partials of its slice), then the rows' norm
// statistics and the bf16 operand. Remote loads of a warp's both rows are in flight before any is used.
__device__ __forceinline__ void PullRows(const LoopDesc& D, float* xf, const float* xs, uint8_t* op, LoopMisc* m,
                                         int nrows, int warp, int lane) {
  const int EB = D.E / kLoopCS, nc = D.E / 8;
  float4 v[2][kLoopMaxChunks][2];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int r = warp + 8 * h;
#pragma unroll
    for (int i = 0; i < kLoopMaxChunks; i++) {
      const int c8 = lane + 32 * i, f = 8 * c8;
      v[h][i][0] = v[h][i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c8 < nc && r < nrows) {
        v[h][i][0] = LdPeer4(PeerAddr(xs + (size_t)r * EB + (f % EB), (uint32_t)(f / EB)));
        v[h][i][1] = LdPeer4(PeerAddr(xs + (size_t)r * EB + ((f + 4) % EB), (uint32_t)((f + 4) / EB)));
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int r = warp + 8 * h;
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < kLoopMaxChunks; i++) {
      const int c8 = lane + 32 * i;
      if (c8 < nc) PutChunk(D, xf, op, r, 8 * c8, v[h][i][0], v[h][i][1], s1, s2);
    }
    RowStatsFromSums(D, m, r, s1, s2, lane);
  }
}

// The end of a layer: this CTA's slice of E / CS features of every row = x + b_proj + the down-projection
// partials [16][E] of every up-tile owner, summed in owner order (all sixteen loads of a float4 in flight).
__device__ __forceinline__ void ReduceDownSlice(const LoopDesc& D, const float* b_proj, const float* xf,
                                                const float* dpart, float* xs, int nrows, int owners, int c) {
  const int EB = D.E / kLoopCS;
  for (int e = threadIdx.x; e < kLoopRows * (EB / 4); e += kLoopThreads) {
    const int r = e / (EB / 4), fi = (e % (EB / 4)) * 4, f = c * EB + fi;
    float4 v[kLoopCS];
    if (r < nrows) {
#pragma unroll
      for (int o = 0; o < kLoopCS; o++)
        v[o] = o < owners ? LdPeer4(PeerAddr(dpart + (size_t)r * D.E + f, (uint32_t)o)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nrows)
#pragma unroll
      for (int o = 0; o < kLoopCS; o++)
        if (o < owners) {
          sum.x += v[o].x; sum.y += v[o].y; sum.z += v[o].z; sum.w += v[o].w;
        }
    const float sv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float b = b_proj != nullptr ? b_proj[f + i] : 0.f;
      xs[(size_t)r * EB + fi + i] = r < nrows ? xf[(size_t)r * D.E + f + i] + (sv[i] + b) : 0.f;
    }
  }
}

// The O reduction of P3 in the same shape: x += the partial O rows of the row's Hk attention items (kv heads in
// order, every CTA alike), then statistics and operand.
__device__ __forceinline__ void ReduceORows(const LoopDesc& D, float* xf, const float* opart, uint8_t* op, LoopMisc* m,
                                            int nrows, int warp, int lane) {
  const int nc = D.E / 8;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int r = warp + 8 * h;
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < kLoopMaxChunks; i++) {
      const int c8 = lane + 32 * i, f = 8 * c8;
      if (c8 >= nc) continue;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (r < nrows) {
        float4 pa[4], pb[4];
        float4 sa = make_float4(0.f, 0.f, 0.f, 0.f), sb = sa;
        for (int g0 = 0; g0 < D.Hk; g0 += 4) {
#pragma unroll
          for (int u = 0; u < 4; u++) {  // up to eight remote loads in flight before the sums
            const int i2 = r * D.Hk + g0 + u;
            if (g0 + u < D.Hk) {
              const float* src = opart + (size_t)(i2 / kLoopCS) * D.E + f;
              pa[u] = LdPeer4(PeerAddr(src, (uint32_t)(i2 % kLoopCS)));
              pb[u] = LdPeer4(PeerAddr(src + 4, (uint32_t)(i2 % kLoopCS)));
            }
          }
#pragma unroll
          for (int u = 0; u < 4; u++)
            if (g0 + u < D.Hk) {
              sa.x += pa[u].x; sa.y += pa[u].y; sa.z += pa[u].z; sa.w += pa[u].w;
              sb.x += pb[u].x; sb.y += pb[u].y; sb.z += pb[u].z; sb.w += pb[u].w;
            }
        }
        a = *reinterpret_cast<const float4*>(xf + (size_t)r * D.E + f);
        b = *reinterpret_cast<const float4*>(xf + (size_t)r * D.E + f + 4);
        a.x += sa.x; a.y += sa.y; a.z += sa.z; a.w += sa.w;
        b.x += sb.x; b.y += sb.y; b.z += sb.z; b.w += sb.w;
      }
      PutChunk(D, xf, op, r, f, a, b, s1, s2);
    }
    RowStatsFromSums(D, m, r, s1, s2, lane);
  }
}

// One decode-attention item (row, kv head) over positions 0..p for the warp's tasks sub, sub + wpi, ...:
// the task layout of AttnRowsKernel (32 positions per task, K/V rows read as coalesced 16-byte chunks).
template <int DD, int MG>
__device__ __forceinline__ void AttendItemWarp(const LoopDesc& D, const float* sq, int layer, int g, int slot, int p,
                                               int sub, int wpi, float* out_state, int lane) {
  constexpr int C = DD / 8, RPI = kAttnTask / C;
  const int ck = lane % C, rg = lane / C;
  const int G = D.G;
  float o[MG][8], mrun[MG], lrun[MG];
#pragma unroll
  for (int h = 0; h < MG; h++) {
    mrun[h] = -INFINITY;
    lrun[h] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) o[h][j] = 0.f;
  }
  const size_t head_off = (size_t)((layer * D.Hk + g) * 2) * kPageTokens * DD;
  const int ntask = p / kAttnTask + 1;
  for (int c = sub; c < ntask; c += wpi) {
    const int t0 = c * kAttnTask;
    const int page = __ldcg(D.kv.block_table + (size_t)slot * D.kv.max_blocks + t0 / kPageTokens);
    if (page < 0) {
      atomicCAS(&g_shahd_device_error, 0, kDevErrNoPage);
      continue;
    }
    const bf16* kb = D.kv.pool + (size_t)page * D.kv.page_elems + head_off + (size_t)(t0 % kPageTokens) * DD;
    const uint4* kp = reinterpret_cast<const uint4*>(kb) + ck;
    const uint4* vp = reinterpret_cast<const uint4*>(kb + (size_t)kPageTokens * DD) + ck;
    uint4 kr[C], vr[C];
#pragma unroll
    for (int i = 0; i < C; i++) {
      const int r = i * RPI + rg;
      if (t0 + r <= p) {
        kr[i] = __ldcg(kp + (size_t)r * C);
        vr[i] = __ldcg(vp + (size_t)r * C);
      } else {
        kr[i] = vr[i] = make_uint4(0, 0, 0, 0);
      }
    }
    const bool valid = t0 + ck * RPI + rg <= p;
    float pv[MG];
#pragma unroll
    for (int h = 0; h < MG; h++) {
      pv[h] = 0.f;
      if (h < G) {
        const float4 q0 = *reinterpret_cast<const float4*>(sq + h * DD + ck * 8);
        const float4 q1 = *reinterpret_cast<const float4*>(sq + h * DD + ck * 8 + 4);
        const float qf[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        float part[C];
#pragma unroll
        for (int i = 0; i < C; i++) {
          float kf[8];
          Bf16ChunkToFloat(kr[i], kf);
          float a = 0.f;
#pragma unroll
          for (int j = 0; j < 8; j++) a = fmaf(qf[j], kf[j], a);
          part[i] = a;
        }
        const float full = ReduceScatter<C>(part, lane);  // every lane takes part in the shuffles
        const float si = valid ? full : -INFINITY;
        const float nm = fmaxf(mrun[h], WarpMax(si));
        const float sc = mrun[h] == -INFINITY ? 0.f : __expf(mrun[h] - nm);
        pv[h] = valid ? __expf(si - nm) : 0.f;
        lrun[h] = lrun[h] * sc + pv[h];
#pragma unroll
        for (int j = 0; j < 8; j++) o[h][j] *= sc;
        mrun[h] = nm;
      }
    }
#pragma unroll
    for (int i = 0; i < C; i++) {
      float vf[8];
      Bf16ChunkToFloat(vr[i], vf);
#pragma unroll
      for (int h = 0; h < MG; h++) {
        if (h < G) {
          const float pt = __shfl_sync(0xffffffffu, pv[h], rg * C + i);
#pragma unroll
          for (int j = 0; j < 8; j++) o[h][j] = fmaf(pt, vf[j], o[h][j]);
        }
      }
    }
  }
  // state: [G] max, [G] sum, [G][DD] unnormalized output (row groups summed)
#pragma unroll
  for (int h = 0; h < MG; h++) {
    if (h < G) {
#pragma unroll
      for (int j = 0; j < 8; j++)
#pragma unroll
        for (int off = C; off < 32; off *= 2) o[h][j] += __shfl_xor_sync(0xffffffffu, o[h][j], off);
      const float l = WarpSum(lrun[h]);
      if (lane == 0) {
        out_state[h] = mrun[h];
        out_state[G + h] = l;
      }
      if (rg == 0) {
#pragma unroll
        for (int j = 0; j < 8; j++) out_state[2 * G + h * DD + ck * 8 + j] = o[h][j];
      }
    }
  }
}

// Lane 0 of warp 0 issues a phase's MMAs (and tops up the weight ring) while lanes 1-31 wait at the warp
// barrier instead of polling the MMA barrier beside it: polling lanes of the same warp would take issue
// slots and suspension time from the one lane the whole cluster is waiting for.
#define ISSUE_PHASE(...)       \
  do {                         \
    if (lane == 0) IssuePhase(__VA_ARGS__); \
    __syncwarp();              \
  } while (0)

// Optional per-phase timestamps (globaltimer, ns) of thread 0 of CTA 0 of cluster 0, one row of kLoopMarks
// per step; D.trace == nullptr (the default) records nothing.
constexpr int kLoopMarks = 22;
#define LOOP_VAL(step, layer, k, v)                                                                        \
  do {                                                                                                     \
    if (D.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0 && (step) < D.trace_steps)               \
      D.trace[((size_t)(step) * (D.L + 1) + (layer)) * kLoopMarks + (k)] = (v);                           \
  } while (0)
#define LOOP_MARK(step, layer, k)                                                                          \
  do {                                                                                                     \
    if (D.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0 && (step) < D.trace_steps)               \
      D.trace[((size_t)(step) * (D.L + 1) + (layer)) * kLoopMarks + (k)] = GlobalTimerNs();                 \
  } while (0)

template <int DD, int MG>
__global__ void __launch_bounds__(kLoopThreads, 1) DecodeLoopKernel(const __grid_constant__ LoopDesc D) {
  extern __shared__ uint8_t loop_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(loop_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* xb = smem + D.off_xb;
  uint8_t* ctxb = smem + D.off_ctxb;
  uint8_t* actb = smem + D.off_actb;
  float* xf = reinterpret_cast<float*>(smem + D.off_xf);
  float* qkv = reinterpret_cast<float*>(smem + D.off_qkv);      // [nq][16][128]
  float* opart = reinterpret_cast<float*>(smem + D.off_opart);  // [items][E]
  float* dpart = reinterpret_cast<float*>(smem + D.off_dpart);  // [16][E]
  float* xs = reinterpret_cast<float*>(smem + D.off_xs);        // [16][E / CS]
  float* att = reinterpret_cast<float*>(smem + D.off_att);      // [entries][2G + G*DD]
  float* sq = reinterpret_cast<float*>(smem + D.off_sq);        // [items][G][DD]
  float* rope = reinterpret_cast<float*>(smem + D.off_rope);    // [2][16 rows][DD / 2]: this step's cos, sin
  LoopMisc* m = reinterpret_cast<LoopMisc*>(smem + D.off_misc);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = (int)ClusterRank();
  const int cluster = blockIdx.x / kLoopCS;
  const int r0 = cluster * D.rows;
  const int nrows = max(0, min(D.rows, D.M - r0));
  const int n_items = LoopCount(nrows * D.Hk, c);  // items i = c + j*CS, row i / Hk, kv head i % Hk
  const int g_item = c % D.Hk;                     // the same for all items of this CTA (CS % Hk == 0)
  const int hd = D.H * DD;
  const int G = D.G;
  const int state_len = 2 * G + G * DD;

  LoopCtx X{D, MakeSched(D, c, n_items), m, ring, c, g_item};
  X.total = D.steps * X.S.per_step;
  X.cons = X.iss = 0;
  X.cst = X.ist = 0;
  X.cpar = X.ipar = 0;
  X.cur = SchedCursor{0, 0, 0, 0, 0, 0};
  if (X.total > 0) SkipEmpty(X.S, D.L, X.cur);
  X.sched = reinterpret_cast<const LoopStage*>(smem + D.off_sched);
  X.sidx = 0;
  X.mma_phase = 0;
  X.wait_full_ns = X.wait_mma_ns = X.issue_ns = X.topup_ns = 0;
  X.blocking_topups = 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < D.stages; s++) {
      MbarInit(&m->full[s], 1);
      MbarInit(&m->empty[s], 1);
    }
    MbarInit(&m->mma_bar, 1);
    m->abort = 0;
    m->issued = 0;
    FenceMbarInit();
    for (int i = 0; i < 4 * D.L + 1; i++) PrefetchTmaDesc(&D.wmaps[i]);
  }
  if (threadIdx.x < kLoopRows) {
    const int r = threadIdx.x;
    if (r < nrows) {
      const int sl = D.slot[r0 + r];
      m->slot[r] = sl;
      m->pos[r] = D.seq_len[sl];
      m->tok[r] = D.tok[r0 + r];
    } else {
      m->slot[r] = 0;
      m->pos[r] = 0;
      m->tok[r] = 0;
    }
  }
  // operand padding stays zero for the whole launch
  for (int i = threadIdx.x; i < (D.off_xf - D.off_xb) / 16; i += kLoopThreads)
    reinterpret_cast<uint4*>(xb)[i] = make_uint4(0, 0, 0, 0);
  __syncwarp();
  if (warp == 0) {
    TmemAlloc(&m->tmem, kLoopTmemCols);
    TmemRelinquish();
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  if (threadIdx.x == 0 && X.total > 0) {
    BuildStageTable(X, reinterpret_cast<LoopStage*>(smem + D.off_sched));
    TopUp(X, false);  // the first weight stages stream in during the embedding
  }
  EmbedRows(D, xf, xb, m, nrows, warp, lane);
  FenceProxyAsyncShared();
  LoopBarrier();  // every CTA of the cluster is running before any remote access

  // Epilogues: warp w reads TMEM lane quadrant w % 4 (output features fl of a 128-feature tile) and the
  // accumulator columns of rows (or items) 8 * rh .. 8 * rh + 7.
  const int quad = warp & 3, rh = warp >> 2;
  const int fl = quad * 32 + lane;
  const uint32_t tq = m->tmem + ((uint32_t)(quad * 32) << 16) + 8u * (uint32_t)rh;

  for (int s = 0; s < D.steps; s++) {
    if (threadIdx.x < kLoopRows) {  // page of the step's position (the host assigned pages for the run)
      const int r = threadIdx.x;
      m->page[r] = r < nrows ? __ldcg(D.kv.block_table + (size_t)m->slot[r] * D.kv.max_blocks + m->pos[r] / kPageTokens) : -1;
    }
    if (D.rope_cos != nullptr)  // the rows' RoPE angles of this step, read by every layer's QKV epilogue
      for (int e = threadIdx.x; e < kLoopRows * (DD / 2); e += kLoopThreads) {
        const int r = e / (DD / 2), i = e % (DD / 2);
        const size_t at = (size_t)(r < nrows ? m->pos[r] : 0) * (DD / 2) + i;
        rope[e] = __ldg(D.rope_cos + at);
        rope[kLoopRows * (DD / 2) + e] = __ldg(D.rope_sin + at);
      }
    for (int l = 0; l < D.L; l++) {
      const LoopLayer ly = D.layers[l];
      LOOP_MARK(s, l, 0);
      // ---------------- P1: gather x, norm1 statistics, QKV + RoPE + KV append ----------------
      if (l > 0) PullRows(D, xf, xs, xb, m, nrows, warp, lane);  // layer 0: from the embedding
      LOOP_MARK(s, l, 1);
      FenceProxyAsyncShared();
      __syncthreads();
      LOOP_MARK(s, l, 2);
      if (warp >= 4) {  // this layer's cached K/V rows of the CTA's attention items into L2
        for (int j = warp - 4; j < n_items; j += kLoopWarps - 4) {
          const int i = c + j * kLoopCS, r = i / D.Hk;
          const int np = m->pos[r] / kPageTokens + 1;
          for (int pg = lane; pg < np; pg += 32) {
            const int page = __ldcg(D.kv.block_table + (size_t)m->slot[r] * D.kv.max_blocks + pg);
            if (page >= 0)
              PrefetchBulkL2(D.kv.pool + (size_t)page * D.kv.page_elems + (size_t)((l * D.Hk + g_item) * 2) * kPageTokens * DD,
                             2u * kPageTokens * DD * 2u);
          }
        }
      }
      if (X.S.nq > 0) {
        if (warp == 0) ISSUE_PHASE(X, X.S.bq, X.S.nkE, kTmQkv, SmemAddr(xb), 64);
        WaitMma(X);
        LOOP_MARK(s, l, 3);
        if (!m->abort) {
          for (int q = 0; q < X.S.nq; q++) {
            const int f = (c + q * kLoopCS) * 128 + fl;
            uint32_t u[8];
            TmemLoad8(tq + kTmQkv + 16u * q, u);
            TmemWaitLd();
            const bool fok = f < D.Nqkv;
            const float c1 = (D.norm == kNormLayer && fok) ? ly.qkv_c1[f] : 0.f;
            const float c2 = (D.norm == kNormLayer && fok) ? ly.qkv_c2[f] : 0.f;
            const bool rope_f = D.rope_cos != nullptr && f < (D.H + D.Hk) * DD;
            const int j = f % DD;
#pragma unroll
            for (int jr = 0; jr < 8; jr++) {
              const int r = 8 * rh + jr;
              float v = __uint_as_float(u[jr]);
              v = D.norm == kNormLayer ? m->is[r] * (v - m->mu[r] * c1) + c2 : v * m->is[r];
              const float partner = __shfl_xor_sync(0xffffffffu, v, 1);  // RoPE pair (2i, 2i+1)
              if (r >= nrows || !fok) continue;
              const int p = m->pos[r];
              if (rope_f) {
                const float cs = rope[r * (DD / 2) + (j >> 1)];
                const float sn = rope[kLoopRows * (DD / 2) + r * (DD / 2) + (j >> 1)];
                v = (j & 1) ? partner * sn + v * cs : v * cs - partner * sn;
              }
              if (f < hd) {
                qkv[((size_t)q * kLoopRows + r) * 128 + fl] = v;
              } else {
                const int kvsel = f < hd + D.Hk * DD ? 0 : 1;
                const int g2 = (f - hd - kvsel * D.Hk * DD) / DD;
                const int page = m->page[r];
                if (page >= 0)
                  D.kv.pool[(size_t)page * D.kv.page_elems +
                            ((size_t)((l * D.Hk + g2) * 2 + kvsel) * kPageTokens + (p & (kPageTokens - 1))) * DD + j] =
                      __float2bfloat16_rn(v);
                else
                  atomicCAS(&g_shahd_device_error, 0, kDevErrNoPage);
              }
            }
          }
        }
      }
      if (threadIdx.x == 0) TopUp(X, false);
      LOOP_MARK(s, l, 4);
      TcgenFenceBefore();
      LoopBarrier();
      TcgenFenceAfter();
      LOOP_MARK(s, l, 5);
      // ---------------- P2: attention of this CTA's items, then their partial O rows ----------------
      for (int e = threadIdx.x; e < n_items * G * DD; e += kLoopThreads) {
        const int jj = e / (G * DD), hf = e % (G * DD);
        const int r = (c + jj * kLoopCS) / D.Hk;
        const int f = g_item * G * DD + hf;  // q feature of head g*G + hf / DD
        const int t = f / 128;
        sq[e] = LdPeer(PeerAddr(qkv + ((size_t)(t / kLoopCS) * kLoopRows + r) * 128 + (f % 128), (uint32_t)(t % kLoopCS))) *
                D.scale;
      }
      __syncthreads();
      {
        const int wpi = n_items > 0 ? max(1, kLoopWarps / n_items) : 1;
        const int groups = kLoopWarps / wpi;
        const int grp = warp / wpi, sub = warp % wpi;
        for (int jj = grp; jj < n_items && grp < groups; jj += groups) {
          const int r = (c + jj * kLoopCS) / D.Hk;
          if (!m->abort)
            AttendItemWarp<DD, MG>(D, sq + (size_t)jj * G * DD, l, g_item, m->slot[r], m->pos[r], sub, wpi,
                                   att + (size_t)(jj * wpi + sub) * state_len, lane);
        }
        __syncthreads();
        // merge the warps of each item; the context rows become the O operand (item slot = operand row)
        for (int e = threadIdx.x; e < n_items * G * DD; e += kLoopThreads) {
          const int jj = e / (G * DD), h = (e % (G * DD)) / DD, dd = e % DD;
          float M = -INFINITY;
          for (int w = 0; w < wpi; w++) M = fmaxf(M, att[(size_t)(jj * wpi + w) * state_len + h]);
          float Ls = 0.f, acc = 0.f;
          for (int w = 0; w < wpi; w++) {
            const float* st = att + (size_t)(jj * wpi + w) * state_len;
            if (st[h] != -INFINITY) {
              const float sc = __expf(st[h] - M);
              Ls += sc * st[G + h];
              acc += sc * st[2 * G + h * DD + dd];
            }
          }
          *reinterpret_cast<bf16*>(ctxb + OpOffset(jj, h * DD + dd)) = __float2bfloat16_rn(Ls > 0.f ? acc / Ls : 0.f);
        }
      }
      FenceProxyAsyncShared();
      __syncthreads();
      LOOP_MARK(s, l, 6);
      if (X.S.no > 0) {
        const int kgd = G * DD - (X.S.nkG - 1) * 64;  // valid K of the last k-block
        if (warp == 0) ISSUE_PHASE(X, X.S.bo, X.S.nkG, kTmO, SmemAddr(ctxb), kgd);
        WaitMma(X);
        LOOP_MARK(s, l, 7);
        if (!m->abort && 8 * rh < n_items) {
          for (int mt = 0; mt < X.S.nE128; mt++) {
            const int f = mt * 128 + fl;
            uint32_t u[8];
            TmemLoad8(tq + kTmO + 16u * mt, u);
            TmemWaitLd();
            if (f < D.E)
#pragma unroll
              for (int jr = 0; jr < 8; jr++)
                if (8 * rh + jr < n_items) opart[(size_t)(8 * rh + jr) * D.E + f] = __uint_as_float(u[jr]);
          }
        }
      }
      if (threadIdx.x == 0) TopUp(X, false);
      LOOP_MARK(s, l, 8);
      TcgenFenceBefore();
      LoopBarrier();
      TcgenFenceAfter();
      LOOP_MARK(s, l, 9);
      // ---------------- P3: O reduction + residual (every CTA, all rows), norm2, MLP up, partial down ----------
      ReduceORows(D, xf, opart, xb, m, nrows, warp, lane);
      LOOP_MARK(s, l, 10);
      FenceProxyAsyncShared();
      __syncthreads();
      LOOP_MARK(s, l, 11);
      if (X.S.nu > 0) {
        if (warp == 0) ISSUE_PHASE(X, X.S.bu, X.S.nkE, kTmUp, SmemAddr(xb), 64);
        WaitMma(X);
        LOOP_MARK(s, l, 12);
        if (!m->abort) {
          for (int uu = 0; uu < X.S.nu; uu++) {
            const int f = (c + uu * kLoopCS) * 128 + fl;
            uint32_t u[8];
            TmemLoad8(tq + kTmUp + 16u * uu, u);
            TmemWaitLd();
            const bool fok = f < D.Nup;
            const float c1 = (D.norm == kNormLayer && fok) ? ly.up_c1[f] : 0.f;
            const float c2 = (D.norm == kNormLayer && fok) ? ly.up_c2[f] : 0.f;
            const float bfc = (D.mlp_kind == 0 && fok) ? ly.b_fc[f] : 0.f;
#pragma unroll
            for (int jr = 0; jr < 8; jr++) {
              const int r = 8 * rh + jr;
              float v = __uint_as_float(u[jr]);
              v = D.norm == kNormLayer ? m->is[r] * (v - m->mu[r] * c1) + c2 : v * m->is[r];
              const float partner = __shfl_xor_sync(0xffffffffu, v, 1);  // gate (even) / up (odd) pair
              if (D.mlp_kind == 0) {
                const float h = (r < nrows && fok) ? fmaxf(v + bfc, 0.f) : 0.f;
                *reinterpret_cast<bf16*>(actb + (size_t)uu * 2 * kLoopOpBlock + OpOffset(r, fl)) = __float2bfloat16_rn(h);
              } else if ((fl & 1) == 0) {
                const float a = GateAct(v, D.mlp_kind == 2);  // GeluValue (Gelu.ts:7-14) / SiluValue (Silu.ts:8-10)
                const float h = (r < nrows && fok) ? a * partner : 0.f;
                *reinterpret_cast<bf16*>(actb + (size_t)uu * kLoopOpBlock + OpOffset(r, fl >> 1)) = __float2bfloat16_rn(h);
              }
            }
          }
        }
        FenceProxyAsyncShared();
        __syncthreads();
        LOOP_MARK(s, l, 13);
        if (warp == 0) ISSUE_PHASE(X, X.S.bd, X.S.nu * X.S.akb, kTmDown, SmemAddr(actb), 64);
        WaitMma(X);
        LOOP_MARK(s, l, 14);
        if (!m->abort) {
          for (int mt = 0; mt < X.S.nE128; mt++) {
            const int f = mt * 128 + fl;
            uint32_t u[8];
            TmemLoad8(tq + kTmDown + 16u * mt, u);
            TmemWaitLd();
            if (f < D.E)
#pragma unroll
              for (int jr = 0; jr < 8; jr++) dpart[(size_t)(8 * rh + jr) * D.E + f] = __uint_as_float(u[jr]);
          }
        }
      }
      if (threadIdx.x == 0) TopUp(X, false);
      LOOP_MARK(s, l, 15);
      TcgenFenceBefore();
      LoopBarrier();
      TcgenFenceAfter();
      LOOP_MARK(s, l, 16);
      // ---------------- P4: this CTA's slice of features: down partials of every up-tile owner + residual ------
      ReduceDownSlice(D, D.mlp_kind == 0 ? ly.b_proj : nullptr, xf, dpart, xs, nrows,
                      min(kLoopCS, CeilDiv(D.Nup, 128)), c);
      if (threadIdx.x == 0) TopUp(X, false);
      LOOP_VAL(s, l, 17, X.wait_full_ns);
      LOOP_VAL(s, l, 18, X.wait_mma_ns);
      LOOP_VAL(s, l, 19, (unsigned long long)(X.iss - X.cons));
      LOOP_VAL(s, l, 20, X.issue_ns);
      LOOP_VAL(s, l, 21, X.topup_ns);
      LoopBarrier();
    }
    // ---------------- head: final norm, LM head tiles, per-row argmax candidates ----------------
    LOOP_MARK(s, D.L, 0);
    PullRows(D, xf, xs, xb, m, nrows, warp, lane);
    FenceProxyAsyncShared();
    __syncthreads();
    {
      float bv[8];
      int bi[8];
#pragma unroll
      for (int jr = 0; jr < 8; jr++) {
        bv[jr] = -INFINITY;
        bi[jr] = 0x7fffffff;
      }
      for (int h0 = 0; h0 < X.S.nh; h0 += kLoopHeadChunk) {
        const int nchunk = min(kLoopHeadChunk, X.S.nh - h0);
        if (warp == 0) ISSUE_PHASE(X, nchunk * X.S.nkE, X.S.nkE, kTmHead, SmemAddr(xb), 64);
        WaitMma(X);
        if (!m->abort) {
          for (int hh = 0; hh < nchunk; hh++) {
            const int vid = (c + (h0 + hh) * kLoopCS) * 128 + fl;
            uint32_t u[8];
            TmemLoad8(tq + kTmHead + 16u * hh, u);
            TmemWaitLd();
            if (vid < D.V) {
              const float c1 = D.norm == kNormLayer ? D.head_c1[vid] : 0.f;
              const float c2 = D.norm == kNormLayer ? D.head_c2[vid] : 0.f;
              const float b = D.head_bias[vid];
#pragma unroll
              for (int jr = 0; jr < 8; jr++) {
                const int r = 8 * rh + jr;
                float v = __uint_as_float(u[jr]);
                v = (D.norm == kNormLayer ? m->is[r] * (v - m->mu[r] * c1) + c2 : v * m->is[r]) + b;
                ArgmaxMerge(bv[jr], bi[jr], v, vid);
                if (D.logits && r < nrows) D.logits[((size_t)(r0 + r) * D.out_ld + D.gen0 + s) * D.V + vid] = v;
              }
            }
          }
        }
        TcgenFenceBefore();
        __syncthreads();  // TMEM chunk read before the next chunk's MMAs overwrite it
        TcgenFenceAfter();
      }
      {
#pragma unroll
        for (int jr = 0; jr < 8; jr++) {
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv[jr], off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi[jr], off);
            ArgmaxMerge(bv[jr], bi[jr], ov, oi);
          }
          if (lane == 0) {
            m->wcv[quad][8 * rh + jr] = bv[jr];
            m->wci[quad][8 * rh + jr] = bi[jr];
          }
        }
      }
      __syncthreads();
      if (threadIdx.x < kLoopRows) {
        const int r = threadIdx.x;
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int w = 0; w < 4; w++) ArgmaxMerge(v, i, m->wcv[w][r], m->wci[w][r]);
        m->cand_v[r] = v;
        m->cand_i[r] = i;
      }
    }
    LOOP_MARK(s, D.L, 1);
    if (threadIdx.x == 0) TopUp(X, false);
    LoopBarrier();
    LOOP_MARK(s, D.L, 2);
    // every CTA: merge the candidates of all CTAs, emit ids, embed them for the next step
    if (threadIdx.x < kLoopRows) {
      const int r = threadIdx.x;
      if (r < nrows) {
        float cv[kLoopCS];
        int ci[kLoopCS];
#pragma unroll
        for (int o = 0; o < kLoopCS; o++) {
          cv[o] = LdPeer(PeerAddr(&m->cand_v[r], (uint32_t)o));
          ci[o] = LdPeerI(PeerAddr(&m->cand_i[r], (uint32_t)o));
        }
        float v = -INFINITY;
        int i = 0x7fffffff;
#pragma unroll
        for (int o = 0; o < kLoopCS; o++) ArgmaxMerge(v, i, cv[o], ci[o]);
        const int id = i == 0x7fffffff ? 0 : i;
        if (c == 0) D.out_ids[(size_t)(r0 + r) * D.out_ld + D.gen0 + s] = id;
        m->tok[r] = id;
        m->pos[r] += 1;
      }
    }
    __syncthreads();
    if (s + 1 < D.steps) EmbedRows(D, xf, xb, m, nrows, warp, lane);
    LOOP_MARK(s, D.L, 3);
  }
  // write the rows' state back (the host's view of the decode loop continues from here)
  if (c == 0 && threadIdx.x < nrows) {
    const int r = threadIdx.x;
    D.tok[r0 + r] = m->tok[r];
    D.seq_len[m->slot[r]] = m->pos[r];
    D.gen_count[r0 + r] += D.steps;
  }
  // drain: loads issued but never consumed (only after an abort) must land before the CTA exits
  if (threadIdx.x == 0) {
    for (int b = X.cons; b < X.iss; b++)
      MbarWaitBounded(&m->full[b % D.stages], (b / D.stages) & 1, kWaitLimit);
  }
  TcgenFenceBefore();
  __syncthreads();
  LoopBarrier();  // no peer reads this CTA's shared memory any more
  if (warp == 0) TmemDealloc(m->tmem, kLoopTmemCols);
}

}  // namespace shahd
