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
constexpr int kLoopStageBytes = 128 * 64 * 2;  // one weight k-block: 128 rows x 64 bf16
constexpr int kLoopOpBlock = kLoopRows * 128;  // one operand k-block: 16 rows x 64 bf16, swizzled
constexpr int kLoopTmemCols = 512;
constexpr int kTmQkv = 0, kTmO = 64, kTmUp = 128, kTmDown = 192, kTmHead = 256;
constexpr int kLoopMaxTiles = 4;   // QKV / up tiles of one CTA, M-tiles of E (64 TMEM columns each region)
constexpr int kLoopHeadChunk = 16; // head tiles per TMEM chunk (256 columns)
constexpr int kLoopMaxStages = 12;

struct LoopLayer {
  const float *qkv_c1, *qkv_c2, *up_c1, *up_c2, *b_fc, *b_proj;
};

// Shapes, pointers and the shared-memory plan of one launch (host-computed, passed by value).
struct LoopDesc {
  int M, E, Ep, H, Hk, d, G, F, Fp, V, L, HDp, Nqkv, Nup;
  int norm, mlp_kind;
  int rows;    // rows per cluster
  int steps;   // decode steps of this launch
  int stages;  // weight ring depth
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
  const CUtensorMap* wmaps;  // [4 L + 1]: qkv, o, up, down of each layer, then the head; box 64 x 128
  // dynamic shared memory plan: byte offsets from the 1024-aligned base
  int off_xb, off_ctxb, off_actb, off_xf, off_qkv, off_opart, off_dpart, off_xs, off_att, off_sq, off_misc;
  int max_items;
  unsigned long long* trace;  // nullable: per-phase timestamps [trace_steps][L + 1][8] (diagnostics)
  int trace_steps;
};

// Host and device agree on the per-CTA work split through these helpers.
__host__ __device__ inline int LoopCount(int total, int rank) { return total > rank ? (total - rank + kLoopCS - 1) / kLoopCS : 0; }
__host__ __device__ inline int LoopActKb(int mlp_kind) { return mlp_kind == 0 ? 2 : 1; }  // act k-blocks per up tile

struct LoopSched {
  int nkE, nkG, nE128, akb;
  int nq, no, nu, nh;      // tiles / M-tiles per phase of this CTA
  int bq, bo, bu, bd, bh;  // weight blocks per phase
  int per_layer, per_step;
};

__device__ __forceinline__ LoopSched MakeSched(const LoopDesc& D, int c, int n_items) {
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
  S.per_layer = S.bq + S.bo + S.bu + S.bd;
  S.per_step = D.L * S.per_layer + S.bh;
  return S;
}

// Weight block b of this CTA's static schedule: tensor map index and box coordinates.
__device__ __forceinline__ void BlockCoords(const LoopDesc& D, const LoopSched& S, int c, int g_item, int b, int& map,
                                            int& x, int& y) {
  const int rem = b % S.per_step;
  if (rem >= D.L * S.per_layer) {  // LM head: tile c + h*CS, k-block kb
    const int i = rem - D.L * S.per_layer;
    map = 4 * D.L;
    x = (i % S.nkE) * 64;
    y = (c + (i / S.nkE) * kLoopCS) * 128;
    return;
  }
  const int l = rem / S.per_layer;
  int i = rem % S.per_layer;
  if (i < S.bq) {
    map = 4 * l;
    x = (i % S.nkE) * 64;
    y = (c + (i / S.nkE) * kLoopCS) * 128;
    return;
  }
  i -= S.bq;
  if (i < S.bo) {  // Wo rows mt, input columns of this CTA's head group
    map = 4 * l + 1;
    x = g_item * D.G * D.d + (i % S.nkG) * 64;
    y = (i / S.nkG) * 128;
    return;
  }
  i -= S.bo;
  if (i < S.bu) {
    map = 4 * l + 2;
    x = (i % S.nkE) * 64;
    y = (c + (i / S.nkE) * kLoopCS) * 128;
    return;
  }
  i -= S.bu;  // W_down rows mt, the input columns of up tile u's activations
  const int per_mt = S.nu * S.akb;
  const int mt = i / per_mt, u = (i % per_mt) / S.akb, kb2 = i % S.akb;
  const int t = c + u * kLoopCS;
  map = 4 * l + 3;
  x = t * 64 * S.akb + kb2 * 64;
  y = mt * 128;
}

// Byte offset of element (row r, column k) of a [16 x K] bf16 operand in 128-byte-swizzled K-major k-blocks.
__device__ __forceinline__ uint32_t OpOffset(int r, int k) {
  return (uint32_t)((k >> 6) * kLoopOpBlock) + Sw128Offset(r, (k & 63) >> 3) + (uint32_t)((k & 7) * 2);
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

__device__ __forceinline__ unsigned long long GlobalTimerNs() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
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
  uint32_t mma_phase;
};

// Thread 0: issue weight loads while ring slots are free (non-blocking), up to `upto` blocks ahead of use.
__device__ __forceinline__ void TopUp(LoopCtx& X, bool block_for_next) {
  const LoopDesc& D = X.D;
  while (X.iss < X.total && X.iss < X.cons + D.stages && !X.m->abort) {
    const int st = X.iss % D.stages;
    const uint32_t ph = ((X.iss / D.stages) & 1) ^ 1;  // the slot's previous use must have been released
    if (X.iss >= D.stages) {
      const bool need = block_for_next && X.iss == X.cons;
      if (need) {
        if (!MbarWaitBounded(&X.m->empty[st], ph, kWaitLimit)) {
          atomicCAS(&g_shahd_device_error, 0, kDevErrLoopTimeout);
          X.m->abort = 1;
          return;
        }
      } else if (!MbarTestWait(&X.m->empty[st], ph)) {
        return;
      }
    }
    int map, x, y;
    BlockCoords(D, X.S, X.c, X.g_item, X.iss, map, x, y);
    MbarArriveExpectTx(&X.m->full[st], kLoopStageBytes);
    TmaLoad2D(X.ring + (size_t)st * kLoopStageBytes, D.wmaps + map, &X.m->full[st], x, y);
    X.iss++;
  }
}

// Thread 0: MMAs of `nblk` consecutive schedule blocks into TMEM columns col0 + 16 * (block / per_tile),
// accumulating over the `per_tile` k-blocks of a tile; `opb(k)` is the operand k-block of schedule block k
// (relative), `kvalid` the valid K of the last k-block of a tile (64 = full). Commits mma_bar at the end.
template <class OpAddr>
__device__ __forceinline__ void IssuePhase(LoopCtx& X, int nblk, int per_tile, uint32_t col0, OpAddr opb, int kvalid_last,
                                           int tile_of_block_div = 0) {
  const uint32_t idesc = UmmaIdescBf16(128, 16);
  for (int k = 0; k < nblk && !X.m->abort; k++) {
    if (X.iss <= X.cons) TopUp(X, true);
    if (X.m->abort) break;
    const int st = X.cons % X.D.stages;
    const uint32_t ph = (X.cons / X.D.stages) & 1;
    if (!MbarWaitBounded(&X.m->full[st], ph, kWaitLimit)) {
      atomicCAS(&g_shahd_device_error, 0, kDevErrLoopTimeout);
      X.m->abort = 1;
      break;
    }
    TcgenFenceAfter();
    const int kin = k % per_tile;
    const int tile = tile_of_block_div > 0 ? k / tile_of_block_div : k / per_tile;
    const uint64_t ad = SmemDescSw128(SmemAddr(X.ring + (size_t)st * kLoopStageBytes));
    const uint64_t bd = SmemDescSw128(opb(k));
    const int kv = (kin == per_tile - 1) ? kvalid_last : 64;
    for (int kk = 0; kk < kv / 16; kk++)
      UmmaBf16(X.m->tmem + col0 + 16u * (uint32_t)tile, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc,
               (kin > 0 || kk > 0) ? 1u : 0u);
    UmmaCommit(&X.m->empty[st]);
    X.cons++;
    TopUp(X, false);
  }
  UmmaCommit(&X.m->mma_bar);  // also completes (vacuously) when nothing was issued
}

// All threads: wait for the phase's MMAs (bounded), then fence for TMEM reads.
__device__ __forceinline__ void WaitMma(LoopCtx& X) {
  const uint32_t ph = X.mma_phase & 1;
  X.mma_phase++;
  if (!MbarWaitBounded(&X.m->mma_bar, ph, kWaitLimit)) {
    atomicCAS(&g_shahd_device_error, 0, kDevErrLoopTimeout);
    X.m->abort = 1;
  }
  TcgenFenceAfter();
}

// Row statistics of the cluster's x rows (NormRow, CachedRowMath.ts:25-56): warp w takes rows w, w + 8.
__device__ __forceinline__ void RowStats(const LoopDesc& D, const float* xf, LoopMisc* m, int warp, int lane) {
  for (int r = warp; r < kLoopRows; r += kLoopWarps) {
    const float* row = xf + (size_t)r * D.E;
    float s1 = 0.f, s2 = 0.f;
    for (int k = lane; k < D.E; k += 32) {
      const float v = row[k];
      s1 += v;
      s2 += v * v;
    }
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
}

// bf16 operand [16 x Ep] from the fp32 rows (padding columns and rows past `nrows` are zero).
__device__ __forceinline__ void BuildOperand(const LoopDesc& D, const float* xf, uint8_t* op, int nrows) {
  const int chunks = D.Ep / 8;
  for (int e = threadIdx.x; e < kLoopRows * chunks; e += kLoopThreads) {
    const int r = e / chunks, k8 = (e % chunks) * 8;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = (r < nrows && k8 + j < D.E) ? xf[(size_t)r * D.E + k8 + j] : 0.f;
    StoreNbf<8>(reinterpret_cast<bf16*>(op + OpOffset(r, k8)), v);
  }
}

// Gathers every owner's slice of E / CS features back into this CTA's x rows.
__device__ __forceinline__ void PullSlices(const LoopDesc& D, float* xf, const float* xs, int nrows) {
  const int EB = D.E / kLoopCS;
  const int n4 = kLoopRows * D.E / 4;
  for (int e = threadIdx.x; e < n4; e += kLoopThreads) {
    const int r = e / (D.E / 4), f = (e % (D.E / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nrows) v = LdPeer4(PeerAddr(xs + (size_t)r * EB + (f % EB), (uint32_t)(f / EB)));
    *reinterpret_cast<float4*>(xf + (size_t)r * D.E + f) = v;
  }
}

// Embeds the rows' current ids (+ learned position) into x (Embedding.ts:14-26).
__device__ __forceinline__ void EmbedRows(const LoopDesc& D, float* xf, const LoopMisc* m, int nrows) {
  for (int e = threadIdx.x; e < kLoopRows * D.E; e += kLoopThreads) {
    const int r = e / D.E, k = e % D.E;
    float v = 0.f;
    if (r < nrows) {
      v = __ldg(D.wte + (size_t)m->tok[r] * D.E + k);
      if (D.wpe) v += __ldg(D.wpe + (size_t)m->pos[r] * D.E + k);
    }
    xf[e] = v;
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
constexpr int kLoopMarks = 8;
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
  float* dpart = reinterpret_cast<float*>(smem + D.off_dpart);  // [E][16]
  float* xs = reinterpret_cast<float*>(smem + D.off_xs);        // [16][E / CS]
  float* att = reinterpret_cast<float*>(smem + D.off_att);      // [entries][2G + G*DD]
  float* sq = reinterpret_cast<float*>(smem + D.off_sq);        // [items][G][DD]
  LoopMisc* m = reinterpret_cast<LoopMisc*>(smem + D.off_misc);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = (int)ClusterRank();
  const int cluster = blockIdx.x / kLoopCS;
  const int r0 = cluster * D.rows;
  const int nrows = max(0, min(D.rows, D.M - r0));
  const int n_items = LoopCount(nrows * D.Hk, c);  // items i = c + j*CS, row i / Hk, kv head i % Hk
  const int g_item = c % D.Hk;                     // the same for all items of this CTA (CS % Hk == 0)
  const int EB = D.E / kLoopCS;
  const int hd = D.H * DD;
  const int G = D.G;
  const int state_len = 2 * G + G * DD;

  LoopCtx X{D, MakeSched(D, c, n_items), m, ring, c, g_item, 0, 0, 0, 0};
  X.total = D.steps * X.S.per_step;

  if (threadIdx.x == 0) {
    for (int s = 0; s < D.stages; s++) {
      MbarInit(&m->full[s], 1);
      MbarInit(&m->empty[s], 1);
    }
    MbarInit(&m->mma_bar, 1);
    m->abort = 0;
    m->issued = 0;
    FenceMbarInit();
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
  if (threadIdx.x == 0) TopUp(X, false);  // the first weight blocks stream in during the embedding
  EmbedRows(D, xf, m, nrows);
  LoopBarrier();  // every CTA of the cluster is running before any remote access

  const int quad = warp & 3;  // TMEM lane quadrant of an epilogue warp (warps 0-3)
  const int fl = quad * 32 + lane;  // tile-local output feature of an epilogue thread
  const uint32_t tq = m->tmem + ((uint32_t)(quad * 32) << 16);

  for (int s = 0; s < D.steps; s++) {
    if (threadIdx.x < kLoopRows) {  // page of the step's position (the host assigned pages for the run)
      const int r = threadIdx.x;
      m->page[r] = r < nrows ? __ldcg(D.kv.block_table + (size_t)m->slot[r] * D.kv.max_blocks + m->pos[r] / kPageTokens) : -1;
    }
    for (int l = 0; l < D.L; l++) {
      const LoopLayer ly = D.layers[l];
      LOOP_MARK(s, l, 0);
      // ---------------- P1: gather x, norm1 statistics, QKV + RoPE + KV append ----------------
      if (l > 0) PullSlices(D, xf, xs, nrows);
      __syncthreads();
      RowStats(D, xf, m, warp, lane);
      BuildOperand(D, xf, xb, nrows);
      FenceProxyAsyncShared();
      __syncthreads();
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
        if (warp == 0) ISSUE_PHASE(X, X.S.bq, X.S.nkE, kTmQkv, [&](int k) { return SmemAddr(xb + (k % X.S.nkE) * kLoopOpBlock); }, 64);
        WaitMma(X);
        if (warp < 4 && !m->abort) {
          for (int q = 0; q < X.S.nq; q++) {
            const int f = (c + q * kLoopCS) * 128 + fl;
            uint32_t u[16];
            TmemLoad16(tq + kTmQkv + 16u * q, u);
            TmemWaitLd();
            const bool fok = f < D.Nqkv;
            const float c1 = (D.norm == kNormLayer && fok) ? ly.qkv_c1[f] : 0.f;
            const float c2 = (D.norm == kNormLayer && fok) ? ly.qkv_c2[f] : 0.f;
            const bool rope = D.rope_cos != nullptr && f < (D.H + D.Hk) * DD;
            const int j = f % DD;
            for (int r = 0; r < kLoopRows; r++) {
              float v = __uint_as_float(u[r]);
              v = D.norm == kNormLayer ? m->is[r] * (v - m->mu[r] * c1) + c2 : v * m->is[r];
              const float partner = __shfl_xor_sync(0xffffffffu, v, 1);  // RoPE pair (2i, 2i+1)
              if (r >= nrows || !fok) continue;
              const int p = m->pos[r];
              if (rope) {
                const float cs = __ldg(D.rope_cos + (size_t)p * (DD / 2) + (j >> 1));
                const float sn = __ldg(D.rope_sin + (size_t)p * (DD / 2) + (j >> 1));
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
      LOOP_MARK(s, l, 1);
      TcgenFenceBefore();
      LoopBarrier();
      TcgenFenceAfter();
      LOOP_MARK(s, l, 2);
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
      LOOP_MARK(s, l, 3);
      if (X.S.no > 0) {
        const int kgd = G * DD - (X.S.nkG - 1) * 64;  // valid K of the last k-block
        if (warp == 0) ISSUE_PHASE(X, X.S.bo, X.S.nkG, kTmO, [&](int k) { return SmemAddr(ctxb + (k % X.S.nkG) * kLoopOpBlock); }, kgd);
        WaitMma(X);
        if (warp < 4 && !m->abort) {
          for (int mt = 0; mt < X.S.nE128; mt++) {
            const int f = mt * 128 + fl;
            uint32_t u[16];
            TmemLoad16(tq + kTmO + 16u * mt, u);
            TmemWaitLd();
            if (f < D.E)
              for (int jj = 0; jj < n_items; jj++) opart[(size_t)jj * D.E + f] = __uint_as_float(u[jj]);
          }
        }
      }
      if (threadIdx.x == 0) TopUp(X, false);
      LOOP_MARK(s, l, 4);
      TcgenFenceBefore();
      LoopBarrier();
      TcgenFenceAfter();
      LOOP_MARK(s, l, 5);
      // ---------------- P3: O reduction + residual (every CTA, all rows), norm2, MLP up, partial down ----------
      for (int e = threadIdx.x; e < nrows * (D.E / 4); e += kLoopThreads) {
        const int r = e / (D.E / 4), f = (e % (D.E / 4)) * 4;
        float4 acc = *reinterpret_cast<float4*>(xf + (size_t)r * D.E + f);
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int g = 0; g < D.Hk; g++) {  // heads in order (the reference sums the per-head projections)
          const int i = r * D.Hk + g;
          const float4 v = LdPeer4(PeerAddr(opart + (size_t)(i / kLoopCS) * D.E + f, (uint32_t)(i % kLoopCS)));
          sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
        }
        acc.x += sum.x; acc.y += sum.y; acc.z += sum.z; acc.w += sum.w;
        *reinterpret_cast<float4*>(xf + (size_t)r * D.E + f) = acc;
      }
      __syncthreads();
      RowStats(D, xf, m, warp, lane);
      BuildOperand(D, xf, xb, nrows);
      FenceProxyAsyncShared();
      __syncthreads();
      if (X.S.nu > 0) {
        if (warp == 0) ISSUE_PHASE(X, X.S.bu, X.S.nkE, kTmUp, [&](int k) { return SmemAddr(xb + (k % X.S.nkE) * kLoopOpBlock); }, 64);
        WaitMma(X);
        if (warp < 4 && !m->abort) {
          for (int uu = 0; uu < X.S.nu; uu++) {
            const int f = (c + uu * kLoopCS) * 128 + fl;
            uint32_t u[16];
            TmemLoad16(tq + kTmUp + 16u * uu, u);
            TmemWaitLd();
            const bool fok = f < D.Nup;
            const float c1 = (D.norm == kNormLayer && fok) ? ly.up_c1[f] : 0.f;
            const float c2 = (D.norm == kNormLayer && fok) ? ly.up_c2[f] : 0.f;
            const float bfc = (D.mlp_kind == 0 && fok) ? ly.b_fc[f] : 0.f;
            for (int r = 0; r < kLoopRows; r++) {
              float v = __uint_as_float(u[r]);
              v = D.norm == kNormLayer ? m->is[r] * (v - m->mu[r] * c1) + c2 : v * m->is[r];
              const float partner = __shfl_xor_sync(0xffffffffu, v, 1);  // gate (even) / up (odd) pair
              if (D.mlp_kind == 0) {
                const float h = (r < nrows && fok) ? fmaxf(v + bfc, 0.f) : 0.f;
                *reinterpret_cast<bf16*>(actb + (size_t)uu * 2 * kLoopOpBlock + OpOffset(r, fl)) = __float2bfloat16_rn(h);
              } else if ((fl & 1) == 0) {
                float a;
                if (D.mlp_kind == 2) {
                  const float cg = 0.7978845608028654f;  // sqrt(2/pi), Gelu.ts:7-14
                  a = 0.5f * v * (1.0f + tanhf(cg * (v + 0.044715f * v * v * v)));
                } else {
                  a = v * (1.0f / (1.0f + __expf(-v)));  // SiluValue, Silu.ts:8-10
                }
                const float h = (r < nrows && fok) ? a * partner : 0.f;
                *reinterpret_cast<bf16*>(actb + (size_t)uu * kLoopOpBlock + OpOffset(r, fl >> 1)) = __float2bfloat16_rn(h);
              }
            }
          }
        }
        FenceProxyAsyncShared();
        __syncthreads();
        if (warp == 0) ISSUE_PHASE(X, X.S.bd, X.S.nu * X.S.akb, kTmDown,
                     [&](int k) { return SmemAddr(actb + (k % (X.S.nu * X.S.akb)) * kLoopOpBlock); }, 64);
        WaitMma(X);
        if (warp < 4 && !m->abort) {
          for (int mt = 0; mt < X.S.nE128; mt++) {
            const int f = mt * 128 + fl;
            uint32_t u[16];
            TmemLoad16(tq + kTmDown + 16u * mt, u);
            TmemWaitLd();
            if (f < D.E)
#pragma unroll
              for (int i = 0; i < 4; i++)
                reinterpret_cast<float4*>(dpart + (size_t)f * kLoopRows)[i] =
                    make_float4(__uint_as_float(u[4 * i]), __uint_as_float(u[4 * i + 1]), __uint_as_float(u[4 * i + 2]),
                                __uint_as_float(u[4 * i + 3]));
          }
        }
      }
      if (threadIdx.x == 0) TopUp(X, false);
      LOOP_MARK(s, l, 6);
      TcgenFenceBefore();
      LoopBarrier();
      TcgenFenceAfter();
      LOOP_MARK(s, l, 7);
      // ---------------- P4: this CTA's slice of features: down partials of every up-tile owner + residual ------
      {
        const int owners = min(kLoopCS, CeilDiv(D.Nup, 128));
        for (int e = threadIdx.x; e < EB * (kLoopRows / 4); e += kLoopThreads) {
          const int fi = e / (kLoopRows / 4), r4 = (e % (kLoopRows / 4)) * 4;
          const int f = c * EB + fi;
          float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int o = 0; o < owners; o++) {
            const float4 v = LdPeer4(PeerAddr(dpart + (size_t)f * kLoopRows + r4, (uint32_t)o));
            sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
          }
          const float b = (D.mlp_kind == 0) ? ly.b_proj[f] : 0.f;
          const float sv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const int r = r4 + i;
            xs[(size_t)r * EB + fi] = r < nrows ? xf[(size_t)r * D.E + f] + (sv[i] + b) : 0.f;
          }
        }
      }
      if (threadIdx.x == 0) TopUp(X, false);
      LoopBarrier();
    }
    // ---------------- head: final norm, LM head tiles, per-row argmax candidates ----------------
    LOOP_MARK(s, D.L, 0);
    PullSlices(D, xf, xs, nrows);
    __syncthreads();
    RowStats(D, xf, m, warp, lane);
    BuildOperand(D, xf, xb, nrows);
    FenceProxyAsyncShared();
    __syncthreads();
    {
      float bv[kLoopRows];
      int bi[kLoopRows];
#pragma unroll
      for (int r = 0; r < kLoopRows; r++) {
        bv[r] = -INFINITY;
        bi[r] = 0x7fffffff;
      }
      for (int h0 = 0; h0 < X.S.nh; h0 += kLoopHeadChunk) {
        const int nchunk = min(kLoopHeadChunk, X.S.nh - h0);
        if (warp == 0) ISSUE_PHASE(X, nchunk * X.S.nkE, X.S.nkE, kTmHead, [&](int k) { return SmemAddr(xb + (k % X.S.nkE) * kLoopOpBlock); },
                     64);
        WaitMma(X);
        if (warp < 4 && !m->abort) {
          for (int hh = 0; hh < nchunk; hh++) {
            const int vid = (c + (h0 + hh) * kLoopCS) * 128 + fl;
            uint32_t u[16];
            TmemLoad16(tq + kTmHead + 16u * hh, u);
            TmemWaitLd();
            if (vid < D.V) {
              const float c1 = D.norm == kNormLayer ? D.head_c1[vid] : 0.f;
              const float c2 = D.norm == kNormLayer ? D.head_c2[vid] : 0.f;
              const float b = D.head_bias[vid];
#pragma unroll
              for (int r = 0; r < kLoopRows; r++) {
                float v = __uint_as_float(u[r]);
                v = (D.norm == kNormLayer ? m->is[r] * (v - m->mu[r] * c1) + c2 : v * m->is[r]) + b;
                ArgmaxMerge(bv[r], bi[r], v, vid);
                if (D.logits && r < nrows) D.logits[((size_t)(r0 + r) * D.out_ld + D.gen0 + s) * D.V + vid] = v;
              }
            }
          }
        }
        TcgenFenceBefore();
        __syncthreads();  // TMEM chunk read before the next chunk's MMAs overwrite it
        TcgenFenceAfter();
      }
      if (warp < 4) {
#pragma unroll
        for (int r = 0; r < kLoopRows; r++) {
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv[r], off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi[r], off);
            ArgmaxMerge(bv[r], bi[r], ov, oi);
          }
          if (lane == 0) {
            m->wcv[warp][r] = bv[r];
            m->wci[warp][r] = bi[r];
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
        float v = -INFINITY;
        int i = 0x7fffffff;
        for (int o = 0; o < kLoopCS; o++)
          ArgmaxMerge(v, i, LdPeer(PeerAddr(&m->cand_v[r], (uint32_t)o)), LdPeerI(PeerAddr(&m->cand_i[r], (uint32_t)o)));
        const int id = i == 0x7fffffff ? 0 : i;
        if (c == 0) D.out_ids[(size_t)(r0 + r) * D.out_ld + D.gen0 + s] = id;
        m->tok[r] = id;
        m->pos[r] += 1;
      }
    }
    __syncthreads();
    if (s + 1 < D.steps) EmbedRows(D, xf, m, nrows);
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
