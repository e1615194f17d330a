// Persistent decode step: every kernel of one batched cached step (embed, L x [QKV + RoPE + KV append,
// attention, O projection + residual, MLP up + activation, MLP down + residual], final norm + LM head) in
// ONE cooperative launch of one CTA per SM (AdvanceOneToken + HeadLogitsRow, CachedForward.ts:32-90 and
// CachedRowMath.ts:117-137, for up to 128 rows).
//
// Why: at decode sizes each of the 33 separate launches of a step moves well under a megabyte but pays
// launch, setup (barriers, TMEM, descriptors) and first-tile latency; the step was bound by that chain.
// Here the phases are separated by a grid-wide barrier (a counter in global memory; every wait is
// bounded), and a CTA issues the weight loads of its next projection tile before it waits at the barrier,
// since weights never depend on the step's data.
//
// Work per phase is a list of items handed out round-robin (item = blockIdx.x + i * gridDim.x):
//   * projection tiles: 128 rows x BN columns (x one K split for the norm-free projections), computed with
//     tcgen05.mma into TMEM by warps 0-3 exactly as the standalone tensor-core kernel does (same operand
//     layout, same epilogue functors);
//   * attention items: one (row, kv head); the CTA's 8 warps take the row's cached pages round-robin,
//     each streaming its page into its own shared buffer with a bulk copy and keeping an online softmax,
//     and the warps' partial results are merged in shared memory.
// The same kernel text serves every layer: per-layer weights are reached through tensor maps kept in
// device memory.
#pragma once

#include "common.cuh"
#include "decode_kernels.cuh"
#include "umma_linear.cuh"

namespace shahd {

constexpr int kStepThreads = 256;  // warps 0-3: tensor-core tiles; all 8 warps: attention pages
constexpr int kStepWarps = kStepThreads / 32;
constexpr int kStepStages = 4;     // k-block stages of the projection tiles
constexpr int kStepBN = 32;        // widest projection tile the stages are sized for
constexpr int kStepMaxD = 64;      // head_dim limit of the per-warp page buffers
constexpr int kStepMaxG = 4;       // query heads per kv head
constexpr int kStepStageBytes = kUmmaBM * kUmmaBK * 2 + kStepBN * kUmmaBK * 2;
constexpr int kStepPageBytes = 2 * kPageTokens * kStepMaxD * 2;  // K + V of one page, per warp
// dynamic shared memory: 1 KB of alignment slack, the projection stages, the per-warp page buffers
constexpr int kStepSmemDyn = 1024 + kStepStages * kStepStageBytes + kStepWarps * kStepPageBytes;
constexpr uint32_t kBarrierSpinLimit = 1u << 24;  // global-barrier polls before a wait gives up

struct StepLayer {
  const float *qkv_c1, *qkv_c2, *up_c1, *up_c2, *b_fc, *b_proj;
};

// Everything one step needs; lives in device memory (pointers and sizes do not change between steps).
struct StepDesc {
  int M, E, Ep, H, Hk, d, G, F, Fp, V, L, HDp, Nqkv, Nup;
  int norm, mlp_kind;
  int bn_qkv, bn_o, bn_up, bn_down, bn_head;  // tile widths (16 or 32)
  int ks_o, ks_down;                           // K splits of the norm-free projections
  int a_box_rows;                              // rows of each activation tile load
  float eps, scale;
  float *x, *q, *ctx, *act, *logits;
  bf16 *xb, *ctxb, *actb;
  int* pos;
  const int *slot, *tok, *seq_len;
  const float *wte, *wpe, *rope_cos, *rope_sin, *head_bias, *head_c1, *head_c2;
  float* am_val;
  int* am_idx;
  KvView kv;
  const StepLayer* layers;
  const CUtensorMap* wmaps;  // [4 L + 1]: per layer qkv, o, up, down; then the LM head
  const CUtensorMap* amaps;  // [3]: xb, ctxb, actb
  float* ws;                 // split-K partial tiles
  int* ws_cnt;               // [N tiles] arrival counters, zero between launches
  unsigned* bar;             // grid barrier counter, zero at launch
  int* abort_flag;           // set when a bounded wait gave up; everything after it is skipped
};

// Per-CTA pipeline state of the projection tiles, identical in every thread of warps 0-3.
struct StepPipe {
  uint64_t* full;   // [kStepStages]
  uint64_t* empty;  // [kStepStages]
  uint64_t* fin;
  uint8_t* stages;
  uint32_t tmem;
  uint32_t kc;       // k-blocks issued so far by this CTA (stage = kc % S, use = kc / S)
  uint32_t fin_phase;
  int prefetched;    // k-blocks of the next tile whose weight loads are already in flight
};

__device__ __forceinline__ bool StepAborted(const StepDesc& s) {
  return *reinterpret_cast<volatile int*>(s.abort_flag) != 0;
}

__device__ __forceinline__ void StepAbort(const StepDesc& s, int code) {
  atomicCAS(&g_shahd_device_error, 0, code);
  atomicExch(s.abort_flag, 1);
}

// Grid-wide barrier: every CTA adds one to the counter and waits for it to reach gen * gridDim.x. The
// wait is bounded; a timeout sets the abort flag so that no CTA waits on the others again.
__device__ __forceinline__ void StepGridBarrier(const StepDesc& s, unsigned& gen) {
  __syncthreads();
  gen += 1;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(s.bar, 1u);
    const unsigned target = gen * gridDim.x;
    bool ok = false;
    for (uint32_t i = 0; i < kBarrierSpinLimit; i++) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(s.bar) : "memory");
      if (v >= target || StepAborted(s)) {
        ok = v >= target;
        break;
      }
    }
    if (!ok) StepAbort(s, kDevErrGemmTimeout);
    __threadfence();
  }
  __syncthreads();
}

// Named barrier of warps 0-3 (the projection warps), leaving warps 4-7 free.
__device__ __forceinline__ void ProjSync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The same barrier, returning whether any of the 128 threads passed true: makes a failure flag uniform
// before code whose barriers every projection thread must reach.
__device__ __forceinline__ bool ProjSyncOr(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}


// Waits until the stage of k-block kk is free (its previous use's MMAs and readers are done). Thread 0.
__device__ __forceinline__ bool StepAcquire(StepPipe& p, uint32_t kk) {
  if (kk < (uint32_t)kStepStages) return true;
  return MbarWaitBounded(&p.empty[kk % kStepStages], (kk / kStepStages - 1) & 1, kWaitLimit);
}

// Weight loads of a tile's first k-blocks, issued before the phase barrier (weights never depend on the
// step's data). Thread 0; the tile then only adds the activation loads of these blocks.
template <int BN>
__device__ __forceinline__ void StepPrefetchW(const StepDesc& s, StepPipe& p, const CUtensorMap* wmap, int n0,
                                              int kb0, int nk) {
  const uint32_t stage_tx = (uint32_t)s.a_box_rows * kUmmaBK * 2 + (uint32_t)BN * kUmmaBK * 2;
  const int n = min(nk, kStepStages);
  int done = 0;
  for (int j = 0; j < n; j++) {
    const uint32_t kk = p.kc + j;
    if (!StepAcquire(p, kk)) {
      StepAbort(s, kDevErrUmmaTimeout);
      break;
    }
    uint8_t* sa = p.stages + (kk % kStepStages) * kStepStageBytes;
    MbarArriveExpectTx(&p.full[kk % kStepStages], stage_tx);
    TmaLoad2D(sa + kUmmaBM * kUmmaBK * 2, wmap, &p.full[kk % kStepStages], (kb0 + j) * kUmmaBK, n0);
    done++;
  }
  p.prefetched = done;
}

// One projection tile (128 rows x BN columns, K split kz of ks) on warps 0-3: the body of the standalone
// tensor-core kernel with the pipeline state carried across tiles. After an abort it only keeps its
// barriers balanced.
template <int NORM, class Epi, int BN>
__device__ __forceinline__ void StepTile(const StepDesc& s, StepPipe& p, const LinearArgs& la, const Epi& epi,
                         const CUtensorMap* wmap, const CUtensorMap* amap, int tile, int ntiles, int kz, int ks,
                         volatile int* s_last) {
  constexpr int S = kStepStages;
  constexpr int kChunks = BN / 16;
  constexpr int kA = kUmmaBM * kUmmaBK * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = threadIdx.x;
  const int n0 = tile * BN;
  const int nk_all = CeilDiv(la.Kp, kUmmaBK);
  const int kb0 = kz * nk_all / ks, nk = (kz + 1) * nk_all / ks - kb0;
  const uint32_t stage_tx = (uint32_t)s.a_box_rows * kUmmaBK * 2 + (uint32_t)BN * kUmmaBK * 2;
  bool fail = ProjSyncOr(StepAborted(s));
  if (threadIdx.x == 0 && fail && p.prefetched > 0) {
    // weight loads issued ahead are still in flight: complete their stages and wait for them (bounded)
    for (int j = 0; j < p.prefetched; j++) {
      const uint32_t kk = p.kc + j;
      TmaLoad2D(p.stages + (kk % S) * kStepStageBytes, amap, &p.full[kk % S], (kb0 + j) * kUmmaBK, 0);
    }
    for (int j = 0; j < p.prefetched; j++) {
      const uint32_t kk = p.kc + j;
      MbarWaitBounded(&p.full[kk % S], (kk / S) & 1, kWaitLimit);
    }
  }
  if (threadIdx.x == 0 && !fail) {
    FenceProxyAsyncGlobal();
    const int n = min(nk, S);
    for (int j = 0; j < n; j++) {
      const uint32_t kk = p.kc + j;
      uint8_t* sa = p.stages + (kk % S) * kStepStageBytes;
      if (j >= p.prefetched) {
        if (!StepAcquire(p, kk)) {
          StepAbort(s, kDevErrUmmaTimeout);
          break;
        }
        MbarArriveExpectTx(&p.full[kk % S], stage_tx);
        TmaLoad2D(sa + kA, wmap, &p.full[kk % S], (kb0 + j) * kUmmaBK, n0);
      }
      TmaLoad2D(sa, amap, &p.full[kk % S], (kb0 + j) * kUmmaBK, 0);
    }
  }
  p.prefetched = 0;
  const bool row_ok = r < la.M;
  const bool vec = epi.vec_ok(la.N);
  typename Epi::Pre pre[kChunks];
  if (vec && row_ok) {
#pragma unroll
    for (int ch = 0; ch < kChunks; ch++)
      if (n0 + 16 * ch + 16 <= la.N) pre[ch] = epi.load16(r, n0 + 16 * ch);
  }
  float s1 = 0.f, s2 = 0.f;
  const uint32_t idesc = UmmaIdescBf16(kUmmaBM, BN);
  for (int kb = 0; kb < nk && !fail; kb++) {
    const uint32_t kk = p.kc + kb;
    const int st = kk % S;
    uint8_t* sa = p.stages + st * kStepStageBytes;
    if (!__all_sync(0xffffffffu, MbarWaitBounded(&p.full[st], (kk / S) & 1, kWaitLimit))) {
      if (lane == 0) StepAbort(s, kDevErrUmmaTimeout);
      fail = true;
      break;
    }
    if (NORM != kNormNone) {
#pragma unroll
      for (int c = 0; c < 8; c++) {
        float f[8];
        Bf16x8ToFloat(*reinterpret_cast<const uint4*>(sa + Sw128Offset(r, c)), f);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          s1 += f[j];
          s2 += f[j] * f[j];
        }
      }
    }
    __syncwarp();
    if (lane == 0) MbarArrive(&p.empty[st]);
    if (threadIdx.x == 0) {
      TcgenFenceAfter();
      const uint64_t ad = SmemDescSw128(SmemAddr(sa));
      const uint64_t bd = SmemDescSw128(SmemAddr(sa + kA));
#pragma unroll
      for (int q = 0; q < kUmmaBK / 16; q++)
        UmmaBf16(p.tmem, ad + (uint64_t)(q * 2), bd + (uint64_t)(q * 2), idesc, (kb > 0 || q > 0) ? 1u : 0u);
      UmmaCommit(&p.empty[st]);
      const int kp = kb - 1;  // refill the previous block's stage with block kp + S
      if (kp >= 0 && kp + S < nk) {
        const uint32_t kkp = p.kc + kp;
        if (!MbarWaitBounded(&p.empty[kkp % S], (kkp / S) & 1, kWaitLimit)) {
          StepAbort(s, kDevErrUmmaTimeout);
        } else {
          uint8_t* sb = p.stages + (kkp % S) * kStepStageBytes;
          MbarArriveExpectTx(&p.full[kkp % S], stage_tx);
          TmaLoad2D(sb, amap, &p.full[kkp % S], (kb0 + kp + S) * kUmmaBK, 0);
          TmaLoad2D(sb + kA, wmap, &p.full[kkp % S], (kb0 + kp + S) * kUmmaBK, n0);
        }
      }
    }
  }
  p.kc += nk;
  if (threadIdx.x == 0 && !fail) UmmaCommit(p.fin);
  float mu = 0.f, is = 1.f;
  if (NORM == kNormRms) {
    is = 1.0f / sqrtf(s2 / la.K + la.eps);
  } else if (NORM == kNormLayer) {
    mu = s1 / la.K;
    is = 1.0f / sqrtf(fmaxf(s2 / la.K - mu * mu, 0.f) + la.eps);
  }
  fail = fail || StepAborted(s);
  if (!__all_sync(0xffffffffu, fail || MbarWaitBounded(p.fin, p.fin_phase, kWaitLimit))) {
    if (lane == 0) StepAbort(s, kDevErrUmmaTimeout);
    fail = true;
  }
  p.fin_phase ^= 1;
  TcgenFenceAfter();
  fail = ProjSyncOr(fail || StepAborted(s));
  const uint32_t trow = p.tmem + ((uint32_t)(warp * 32) << 16);
  bool last = true;
  if (!fail && ks > 1) {
    float* part = la.ws + ((size_t)(tile * ks + kz) * kUmmaBM + r) * BN;
#pragma unroll
    for (int ch = 0; ch < kChunks; ch++) {
      uint32_t u[16];
      TmemLoad16(trow + (uint32_t)(16 * ch), u);
      TmemWaitLd();
      if (row_ok) StoreNf<16>(part + 16 * ch, reinterpret_cast<const float*>(u));
    }
    __threadfence();
    ProjSync();
    if (threadIdx.x == 0) *s_last = atomicAdd(la.ws_cnt + tile, 1) == ks - 1;
    ProjSync();
    last = *s_last != 0;
    if (last) __threadfence();
  }
  if (!fail && last) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int ch = 0; ch < kChunks; ch++) {
      const int nb = n0 + 16 * ch;
      float v[16];
      if (ks > 1) {
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = 0.f;
        if (row_ok) {
          for (int z = 0; z < ks; z++) {
            const float4* src =
                reinterpret_cast<const float4*>(la.ws + ((size_t)(tile * ks + z) * kUmmaBM + r) * BN + 16 * ch);
#pragma unroll
            for (int i = 0; i < 4; i++) {
              const float4 t = __ldcg(src + i);
              v[4 * i] += t.x;
              v[4 * i + 1] += t.y;
              v[4 * i + 2] += t.z;
              v[4 * i + 3] += t.w;
            }
          }
        }
      } else {
        uint32_t u[16];
        TmemLoad16(trow + (uint32_t)(16 * ch), u);
        TmemWaitLd();
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = __uint_as_float(u[j]);
      }
      if (!row_ok) continue;
      if (vec && nb + 16 <= la.N) {
        if (NORM == kNormRms) {
#pragma unroll
          for (int j = 0; j < 16; j++) v[j] *= is;
        } else if (NORM == kNormLayer) {
          float c1[16], c2[16];
          Load16f(la.c1 + nb, c1);
          Load16f(la.c2 + nb, c2);
#pragma unroll
          for (int j = 0; j < 16; j++) v[j] = is * (v[j] - mu * c1[j]) + c2[j];
        }
        epi.store16(r, nb, v, pre[ch]);
        if constexpr (IsLogits<Epi>::value) {
#pragma unroll
          for (int j = 0; j < 16; j++) ArgmaxMerge(bv, bi, v[j], nb + j);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const int n = nb + j;
          if (n < la.N) {
            float v0 = v[j], v1 = v[j + 1];
            if (NORM == kNormRms) {
              v0 *= is;
              v1 *= is;
            } else if (NORM == kNormLayer) {
              v0 = is * (v0 - mu * la.c1[n]) + la.c2[n];
              if (n + 1 < la.N) v1 = is * (v1 - mu * la.c1[n + 1]) + la.c2[n + 1];
            }
            epi.apply(r, n, v0, v1, la.N);
            if constexpr (IsLogits<Epi>::value) {
              ArgmaxMerge(bv, bi, v0, n);
              if (n + 1 < la.N) ArgmaxMerge(bv, bi, v1, n + 1);
            }
          }
        }
      }
    }
    if constexpr (IsLogits<Epi>::value) {
      if (row_ok) {
        la.am_val[(size_t)r * ntiles + tile] = bv;
        la.am_idx[(size_t)r * ntiles + tile] = bi;
      }
    }
    if (ks > 1 && threadIdx.x == 0) la.ws_cnt[tile] = 0;
  }
  TcgenFenceBefore();
  ProjSync();  // TMEM and the stages' readers are done before the next tile's MMAs
}

// Embedding of one decode row (EmbeddingLookup + learned positions, Embedding.ts:14-26): the row's position
// is its slot's cached length.
__device__ __forceinline__ void StepEmbedRow(const StepDesc& s, int r) {
  const int p = s.seq_len[s.slot[r]];
  const int tok = s.tok[r];
  if (threadIdx.x == 0) s.pos[r] = p;
  const float* src = s.wte + (size_t)tok * s.E;
  const float* pe = s.wpe ? s.wpe + (size_t)p * s.E : nullptr;
  for (int j = threadIdx.x; j < s.E; j += blockDim.x) {
    const float v = pe ? src[j] + pe[j] : src[j];
    s.x[(size_t)r * s.E + j] = v;
    s.xb[(size_t)r * s.Ep + j] = __float2bfloat16_rn(v);
  }
}

// Attention of one (row m, kv head g) over positions 0..pos[m] (AttendRow, CachedRowMath.ts:60-86): warp w
// takes pages w, w + 8, ... of the row, streams each (K and V blocks) into its own buffer with bulk copies
// and keeps an online softmax for the group's G query heads; the 8 partial results are merged in shared
// memory. pcnt counts the warp's page loads (the parity of its barrier).
//
// Scores need no shuffles: lane l owns positions l and l + 32 of the page and walks the head dimension
// two at a time starting at word (c + l) mod D/2, so the 32 lanes read 32 different banks of the K rows.
template <int D, int G>
__device__ __forceinline__ void StepAttnItem(const StepDesc& s, int layer, int m, int g, uint8_t* bufs,
                                             uint64_t* pbar, float* sq, float* ss_all, uint32_t& pcnt) {
  constexpr int W2 = D / 2;     // bf16 pairs per K row
  constexpr int JPL = D / 32;   // output dims per lane
  constexpr int PAGE = kPageTokens * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = s.H * D;
  const int p = s.pos[m], slot = s.slot[m];
  const int pages = (p + kPageTokens) / kPageTokens;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) sq[e] = s.q[(size_t)m * hd + g * G * D + e];
  __syncthreads();
  bf16* sk = reinterpret_cast<bf16*>(bufs + warp * kStepPageBytes);
  bf16* sv = sk + PAGE;
  float* ss = ss_all + warp * kStepMaxG * kPageTokens;
  const float scale = s.scale;
  float mloc[G], lloc[G], o[G][JPL];
#pragma unroll
  for (int i = 0; i < G; i++) {
    mloc[i] = -INFINITY;
    lloc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < JPL; j++) o[i][j] = 0.f;
  }
  bool fail = StepAborted(s);
  for (int pg = warp; pg < pages && !fail; pg += kStepWarps) {
    const bool present = s.kv.block_table[slot * s.kv.max_blocks + pg] >= 0;
    const int tv = present ? min(kPageTokens, p + 1 - pg * kPageTokens) : 0;
    if (lane == 0) {
      const bf16* kb = s.kv.Block(slot, pg, layer, g, 0);
      const bf16* vb = s.kv.Block(slot, pg, layer, g, 1);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic smem use before the copy
      if (kb == nullptr || tv == 0) {
        MbarArrive(pbar + warp);
      } else {
        const uint32_t bytes = (uint32_t)tv * D * 2;
        MbarArriveExpectTx(pbar + warp, 2 * bytes);
        BulkCopyG2S(sk, kb, bytes, pbar + warp);
        BulkCopyG2S(sv, vb, bytes, pbar + warp);
      }
    }
    const bool ok = __all_sync(0xffffffffu, MbarWaitBounded(pbar + warp, pcnt & 1, kWaitLimit));
    pcnt++;
    if (!ok) {
      if (lane == 0) StepAbort(s, kDevErrAttnTimeout);
      fail = true;
      break;
    }
    // scores of positions lane and lane + 32 (rows past tv hold stale data and are masked below)
    const __nv_bfloat162* k0 = reinterpret_cast<const __nv_bfloat162*>(sk) + lane * W2;
    const __nv_bfloat162* k1 = k0 + 32 * W2;
    const float2* q2 = reinterpret_cast<const float2*>(sq);
    float a0[G], a1[G];
#pragma unroll
    for (int i = 0; i < G; i++) a0[i] = a1[i] = 0.f;
#pragma unroll 8
    for (int c = 0; c < W2; c++) {
      const int wd = (c + lane) & (W2 - 1);
      const float2 f0 = __bfloat1622float2(k0[wd]), f1 = __bfloat1622float2(k1[wd]);
#pragma unroll
      for (int i = 0; i < G; i++) {
        const float2 qv = q2[i * W2 + wd];
        a0[i] = fmaf(f0.x, qv.x, fmaf(f0.y, qv.y, a0[i]));
        a1[i] = fmaf(f1.x, qv.x, fmaf(f1.y, qv.y, a1[i]));
      }
    }
    // online softmax update per head; the page's weights go to shared memory for the V pass
#pragma unroll
    for (int i = 0; i < G; i++) {
      const float s0 = lane < tv ? a0[i] * scale : -INFINITY;
      const float s1 = lane + 32 < tv ? a1[i] * scale : -INFINITY;
      const float nm = fmaxf(mloc[i], WarpMax(fmaxf(s0, s1)));
      const float e0 = lane < tv ? __expf(s0 - nm) : 0.f;
      const float e1 = lane + 32 < tv ? __expf(s1 - nm) : 0.f;
      ss[i * kPageTokens + lane] = e0;
      ss[i * kPageTokens + lane + 32] = e1;
      const float sum = WarpSum(e0 + e1);
      const float sc = mloc[i] == -INFINITY ? 0.f : __expf(mloc[i] - nm);
      lloc[i] = lloc[i] * sc + sum;
      mloc[i] = nm;
#pragma unroll
      for (int j = 0; j < JPL; j++) o[i][j] *= sc;
    }
    __syncwarp();
    // o += sum_t e_t v_t: lanes over the head dimension, two interleaved partial sums per output
    float ob[G][JPL];
#pragma unroll
    for (int i = 0; i < G; i++)
#pragma unroll
      for (int j = 0; j < JPL; j++) ob[i][j] = 0.f;
#pragma unroll 4
    for (int t = 0; t < tv; t += 2) {
      const bool has_b = t + 1 < tv;  // row tv is stale shared memory: never multiplied, not even by 0
      float va[JPL], vb[JPL];
      if constexpr (JPL == 2) {
        const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sv + t * D + lane * 2));
        const float2 y = has_b ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sv + (t + 1) * D + lane * 2))
                               : make_float2(0.f, 0.f);
        va[0] = x.x; va[1] = x.y; vb[0] = y.x; vb[1] = y.y;
      } else {
#pragma unroll
        for (int j = 0; j < JPL; j++) {
          va[j] = __bfloat162float(sv[t * D + lane * JPL + j]);
          vb[j] = has_b ? __bfloat162float(sv[(t + 1) * D + lane * JPL + j]) : 0.f;
        }
      }
#pragma unroll
      for (int i = 0; i < G; i++) {
        const float ea = ss[i * kPageTokens + t], eb = ss[i * kPageTokens + t + 1];  // 0 past tv
#pragma unroll
        for (int j = 0; j < JPL; j++) {
          o[i][j] = fmaf(ea, va[j], o[i][j]);
          ob[i][j] = fmaf(eb, vb[j], ob[i][j]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < G; i++)
#pragma unroll
      for (int j = 0; j < JPL; j++) o[i][j] += ob[i][j];
    __syncwarp();  // the buffer and the weights are free for the next page
  }
  // the warp's partial (max, sum, output) into its own buffer, then merged across warps in warp order
  float* part = reinterpret_cast<float*>(bufs + warp * kStepPageBytes);  // [G][2 + D]
#pragma unroll
  for (int i = 0; i < G; i++) {
    if (lane == 0) {
      part[i * (D + 2)] = mloc[i];
      part[i * (D + 2) + 1] = lloc[i];
    }
#pragma unroll
    for (int j = 0; j < JPL; j++) part[i * (D + 2) + 2 + lane * JPL + j] = o[i][j];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int i = e / D, j = e % D;
    float mx = -INFINITY;
    for (int w = 0; w < kStepWarps; w++)
      mx = fmaxf(mx, reinterpret_cast<const float*>(bufs + w * kStepPageBytes)[i * (D + 2)]);
    float num = 0.f, den = 0.f;
    for (int w = 0; w < kStepWarps; w++) {
      const float* pw = reinterpret_cast<const float*>(bufs + w * kStepPageBytes) + i * (D + 2);
      const float wt = pw[0] == -INFINITY ? 0.f : __expf(pw[0] - mx);
      num += wt * pw[2 + j];
      den += wt * pw[1];
    }
    const float v = den > 0.f ? num / den : 0.f;
    const int col = (g * G + i) * D + j;
    s.ctx[(size_t)m * hd + col] = v;
    s.ctxb[(size_t)m * s.HDp + col] = __float2bfloat16_rn(v);
  }
  __syncthreads();  // buffers free for the next item
}

// Projection phase descriptors built in the kernel from the step description.
enum StepProj { kProjQkv = 0, kProjO = 1, kProjUp = 2, kProjDown = 3, kProjHead = 4 };

struct StepProjInfo {
  LinearArgs la{};
  const CUtensorMap* wmap;
  const CUtensorMap* amap;
  int bn, ks, tiles;
};

__device__ __forceinline__ StepProjInfo StepProjArgs(const StepDesc& s, int kind, int layer) {
  StepProjInfo pi;
  LinearArgs& la = pi.la;
  la.a = nullptr;
  la.lda = 0;
  la.a_rows = 0;
  la.M = s.M;
  la.w = nullptr;
  la.eps = s.eps;
  la.c1 = la.c2 = nullptr;
  la.am_val = nullptr;
  la.am_idx = nullptr;
  la.ws = nullptr;
  la.ws_cnt = nullptr;
  pi.ks = 1;
  const StepLayer& ly = s.layers[layer];
  switch (kind) {
    case kProjQkv:
      la.ab = s.xb; la.ldab = s.Ep; la.K = s.E; la.Kp = s.Ep; la.N = s.Nqkv; la.c1 = ly.qkv_c1; la.c2 = ly.qkv_c2;
      pi.bn = s.bn_qkv; pi.amap = s.amaps + 0; pi.wmap = s.wmaps + 4 * layer + 0;
      break;
    case kProjO:
      la.ab = s.ctxb; la.ldab = s.HDp; la.K = s.H * s.d; la.Kp = s.HDp; la.N = s.E; la.ws = s.ws; la.ws_cnt = s.ws_cnt;
      pi.bn = s.bn_o; pi.ks = s.ks_o; pi.amap = s.amaps + 1; pi.wmap = s.wmaps + 4 * layer + 1;
      break;
    case kProjUp:
      la.ab = s.xb; la.ldab = s.Ep; la.K = s.E; la.Kp = s.Ep; la.N = s.Nup; la.c1 = ly.up_c1; la.c2 = ly.up_c2;
      pi.bn = s.bn_up; pi.amap = s.amaps + 0; pi.wmap = s.wmaps + 4 * layer + 2;
      break;
    case kProjDown:
      la.ab = s.actb; la.ldab = s.Fp; la.K = s.F; la.Kp = s.Fp; la.N = s.E; la.ws = s.ws; la.ws_cnt = s.ws_cnt;
      pi.bn = s.bn_down; pi.ks = s.ks_down; pi.amap = s.amaps + 2; pi.wmap = s.wmaps + 4 * layer + 3;
      break;
    default:  // LM head
      la.ab = s.xb; la.ldab = s.Ep; la.K = s.E; la.Kp = s.Ep; la.N = s.V; la.c1 = s.head_c1; la.c2 = s.head_c2;
      la.am_val = s.am_val; la.am_idx = s.am_idx;
      pi.bn = s.bn_head; pi.amap = s.amaps + 0; pi.wmap = s.wmaps + 4 * s.L;
      break;
  }
  pi.tiles = CeilDiv(la.N, pi.bn);
  return pi;
}

// Runs this CTA's items of one projection phase (warps 0-3). BN is fixed per phase (16 for the layer
// projections, 32 for the LM head) to keep one copy of the tile code per phase.
template <int NORM, int BN, class Epi>
__device__ __forceinline__ void StepProjPhase(const StepDesc& s, StepPipe& p, const StepProjInfo& pi, const Epi& epi,
                                              volatile int* s_last) {
  const int items = pi.tiles * pi.ks;
  for (int it = blockIdx.x; it < items; it += gridDim.x)
    StepTile<NORM, Epi, BN>(s, p, pi.la, epi, pi.wmap, pi.amap, it / pi.ks, pi.tiles, it % pi.ks, pi.ks, s_last);
}

// Weight loads of this CTA's first tile of a coming projection phase (thread 0), before the barrier.
__device__ __forceinline__ void StepPrefetchPhase(const StepDesc& s, StepPipe& p, const StepProjInfo& pi) {
  if (threadIdx.x != 0 || (int)blockIdx.x >= pi.tiles * pi.ks || StepAborted(s)) return;
  const int tile = blockIdx.x / pi.ks, kz = blockIdx.x % pi.ks;
  const int nk_all = CeilDiv(pi.la.Kp, kUmmaBK);
  const int kb0 = kz * nk_all / pi.ks, nk = (kz + 1) * nk_all / pi.ks - kb0;
  if (pi.bn == 16) StepPrefetchW<16>(s, p, pi.wmap, tile * 16, kb0, nk);
  else StepPrefetchW<32>(s, p, pi.wmap, tile * 32, kb0, nk);
}

template <int NORM, int D>
__global__ void __launch_bounds__(kStepThreads, 1) DecodeStepKernel(const __grid_constant__ StepDesc s) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment by an offset from the shared array itself, so the compiler keeps shared-memory
  // addressing for every pointer derived from it
  uint8_t* base = smem_raw + ((1024u - (SmemAddr(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t bars[2 * kStepStages + 1 + kStepWarps];
  __shared__ uint32_t s_tmem;
  __shared__ int s_last;
  __shared__ __align__(16) float sq[kStepMaxG * kStepMaxD];
  __shared__ float ss_all[kStepWarps * kStepMaxG * kPageTokens];
  const int warp = threadIdx.x >> 5;
  StepPipe p;
  p.full = bars;
  p.empty = bars + kStepStages;
  p.fin = bars + 2 * kStepStages;
  uint64_t* pbar = bars + 2 * kStepStages + 1;
  p.stages = base;
  uint8_t* bufs = base + kStepStages * kStepStageBytes;
  p.kc = 0;
  p.fin_phase = 0;
  p.prefetched = 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStepStages; i++) {
      MbarInit(&p.full[i], 1);
      MbarInit(&p.empty[i], 1 + 4);  // the MMA commit + one arrival per projection warp
    }
    MbarInit(p.fin, 1);
    for (int w = 0; w < kStepWarps; w++) MbarInit(pbar + w, 1);
    FenceMbarInit();
  }
  if (warp == 0) {
    TmemAlloc(&s_tmem, kStepBN);
    TmemRelinquish();
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  p.tmem = s_tmem;
  uint32_t pcnt = 0;
  unsigned gen = 0;

  // embedding rows; meanwhile the first QKV weights are on their way
  StepPrefetchPhase(s, p, StepProjArgs(s, kProjQkv, 0));
  for (int r = blockIdx.x; r < s.M; r += gridDim.x) StepEmbedRow(s, r);
  StepGridBarrier(s, gen);

  for (int l = 0; l < s.L; l++) {
    {  // norm1 + QKV + RoPE + KV append (CachedForward.ts:66-73, :78-79)
      const StepProjInfo pi = StepProjArgs(s, kProjQkv, l);
      const EpiQKV epi{s.q, s.kv, l, s.pos, s.slot, s.rope_cos, s.rope_sin, s.H, s.Hk, s.d};
      if (warp < 4) StepProjPhase<NORM, 16>(s, p, pi, epi, &s_last);
    }
    StepGridBarrier(s, gen);
    {  // attention over the cache (CachedForward.ts:76-80)
      if (threadIdx.x == 0) FenceProxyAsyncGlobal();
      for (int it = blockIdx.x; it < s.M * s.Hk; it += gridDim.x) {
        if (s.G == 1) StepAttnItem<D, 1>(s, l, it / s.Hk, it % s.Hk, bufs, pbar, sq, ss_all, pcnt);
        else if (s.G == 2) StepAttnItem<D, 2>(s, l, it / s.Hk, it % s.Hk, bufs, pbar, sq, ss_all, pcnt);
        else StepAttnItem<D, 4>(s, l, it / s.Hk, it % s.Hk, bufs, pbar, sq, ss_all, pcnt);
      }
      StepPrefetchPhase(s, p, StepProjArgs(s, kProjO, l));
    }
    StepGridBarrier(s, gen);
    {  // summed per-head Wo + residual (CachedForward.ts:81-84)
      const StepProjInfo pi = StepProjArgs(s, kProjO, l);
      const EpiResid epi{s.x, s.xb, s.E, s.Ep, nullptr};
      if (warp < 4) StepProjPhase<kNormNone, 16>(s, p, pi, epi, &s_last);
      StepPrefetchPhase(s, p, StepProjArgs(s, kProjUp, l));
    }
    StepGridBarrier(s, gen);
    {  // norm2 + MLP up (+ activation) (CachedForward.ts:86-87, MlpRow)
      const StepProjInfo pi = StepProjArgs(s, kProjUp, l);
      if (warp < 4) {
        if (s.mlp_kind == 0)
          StepProjPhase<NORM, 16>(s, p, pi, EpiReluFc{s.act, s.actb, s.F, s.Fp, s.layers[l].b_fc}, &s_last);
        else
          StepProjPhase<NORM, 16>(s, p, pi, EpiGated{s.act, s.actb, s.F, s.Fp, s.mlp_kind == 2}, &s_last);
      }
      StepPrefetchPhase(s, p, StepProjArgs(s, kProjDown, l));
    }
    StepGridBarrier(s, gen);
    {  // MLP down + residual
      const StepProjInfo pi = StepProjArgs(s, kProjDown, l);
      const EpiResid epi{s.x, s.xb, s.E, s.Ep, s.layers[l].b_proj};
      if (warp < 4) StepProjPhase<kNormNone, 16>(s, p, pi, epi, &s_last);
      StepPrefetchPhase(s, p, l + 1 < s.L ? StepProjArgs(s, kProjQkv, l + 1) : StepProjArgs(s, kProjHead, 0));
    }
    StepGridBarrier(s, gen);
  }
  {  // final norm + LM head + argmax partials (HeadLogitsRow, CachedRowMath.ts:117-137)
    const StepProjInfo pi = StepProjArgs(s, kProjHead, 0);
    if (warp < 4) StepProjPhase<NORM, 32>(s, p, pi, EpiLogits{s.logits, s.head_bias, s.V}, &s_last);
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  if (warp == 0) TmemDealloc(p.tmem, kStepBN);
}

}  // namespace shahd
