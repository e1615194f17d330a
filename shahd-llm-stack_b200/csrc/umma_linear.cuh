// Tensor-core (tcgen05 / TMEM / TMA) kernels for sm_100a.
//
// LinearUmmaKernel: the batched-rows regime of every decode/prefill projection. 128-row x BN-column
// output tile per CTA; the weight tile [BN x 64] (issued before the grid-dependency wait) and the bf16
// activation rows [up to 128 x 64] arrive by TMA (128-byte swizzle, K-major); the layer norm
// (NormRow, CachedRowMath.ts:25-56) is folded into the weights, its per-row statistics are taken from
// the staged activation tiles and applied in the epilogue; one thread issues tcgen05.mma (M=128, N=BN,
// K=16) into a TMEM accumulator; the four warps read their 32-lane quadrant back with tcgen05.ld and
// run the fused epilogue (RoPE + KV append, residual add, SwiGLU/GeGLU, LM head + argmax). A long
// decode reduction is split over a cluster of CTAs that sum their partial tiles through distributed
// shared memory.
//
// The batched-prefill projections and the MatMulNT operator run the persistent warp-specialized kernel of
// gemm_persist.cuh instead.
//
// Every mbarrier wait is bounded; on timeout the kernel records an error code in g_shahd_device_error,
// skips the remaining work, releases its TMEM and returns.
#pragma once

#include <algorithm>
#include <map>
#include <mutex>

#include "common.cuh"
#include "decode_kernels.cuh"

namespace shahd {

constexpr int kUmmaBM = 128;
constexpr int kUmmaBK = 64;
constexpr int kUmmaThreads = 128;

// Rows at which a projection switches from the SIMT (CUDA-core) kernel to tensor-core tiles. Settable
// through ShahdSetTensorCoreMinRows / SetScalarKernels (test hooks, process-wide).
extern int g_umma_min_rows;
extern int g_decode_chains;
extern int g_persistent_step;
extern int g_umma_prefill_attn;
extern int g_decode_attn_kernel;
#define kUmmaMinRows (::shahd::g_umma_min_rows)

// Tile width: prefill-sized row counts take wide tiles; decode-sized ones the narrowest tile whose grid
// still fits one wave of CTAs (more CTAs stream the weights in parallel, each with a shorter queue).
constexpr int kUmmaWaveCtas = 148;
__host__ inline int UmmaBN(int M, int N) {
  if (M > kUmmaBM) return 128;
  for (int bn = 16; bn <= 64; bn *= 2)
    if (CeilDiv(N, bn) <= kUmmaWaveCtas) return bn;
  return 128;
}

// K splits of a decode-sized projection without a norm (the norm needs whole rows): about four k-blocks
// of 64 per CTA, at most 8 splits (one cluster) and two waves of CTAs. Partial tiles meet in the
// cluster's shared memory; the workspace pointer only marks a projection as splittable.
__host__ inline int UmmaKSplit(int M, int N, int Kp) {
  if (M > kUmmaBM) return 1;
  const int nk = CeilDiv(Kp, kUmmaBK), tiles = CeilDiv(N, UmmaBN(M, N));
  int ks = std::min(8, std::max(1, nk / 4));
  while (ks > 1 && tiles * ks > 2 * kUmmaWaveCtas) ks--;
  return ks;
}
// Workspace floats for split-K partials of an N-column projection (one launch at a time).
__host__ inline size_t UmmaKSplitFloats(int N, int Kp) {
  const int bn = UmmaBN(1, N);
  return (size_t)CeilDiv(N, bn) * bn * UmmaKSplit(1, N, Kp) * kUmmaBM;
}
__host__ inline int UmmaGridN(int N) { return CeilDiv(N, 16); }  // upper bound of N tiles (BN >= 16)

inline bool UmmaLinearSupported(const LinearArgs& la) { return la.Kp % 8 == 0 && la.N >= 1 && la.ab != nullptr; }

// Pipeline depth by tile width: narrow tiles keep a whole decode-sized K in flight.
// Stage ring depth. BN = 128 tiles (batched prefill rows, a few k-blocks each) keep two stages, so three
// CTAs share an SM and one CTA's epilogue overlaps the others' main loops (4096-sequence prefill-heavy
// job 149 -> 134 ms against four stages).
__host__ __device__ constexpr int UmmaStages(int BN) { return BN <= 32 ? 8 : (BN <= 64 ? 6 : 2); }

// Rows of the activation tile fetched per stage: the 8-row multiple covering M (at most 128). The MMA
// always reads 128 rows; the rows past the box hold stale shared memory and only feed accumulator rows
// that are never stored.
__host__ inline int UmmaBoxRows(int M) { return M >= kUmmaBM ? kUmmaBM : RoundUp(M, 8); }

template <int BN>
struct UmmaSmem {
  static constexpr int kStages = UmmaStages(BN);
  static constexpr int kA = kUmmaBM * kUmmaBK * 2;  // 16 KB
  static constexpr int kB = BN * kUmmaBK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kBytes = kStages * kStage + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
};

// ---- host: TMA descriptor for a bf16 row-major [rows, cols] matrix, box [box_rows, 64] ------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn GetEncodeTiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Cached per (pointer, shape, box): weights are fixed for a session's lifetime, and a session forgets its own
// entries when it frees its memory (ForgetTmaRange), so the cache holds only live buffers.
struct TmaKey {
  const void* p;
  int r, c, ld, b;
  bool operator<(const TmaKey& o) const {
    if (p != o.p) return p < o.p;
    if (r != o.r) return r < o.r;
    if (c != o.c) return c < o.c;
    if (ld != o.ld) return ld < o.ld;
    return b < o.b;
  }
};
inline std::mutex& TmaCacheMutex() {
  static std::mutex mu;
  return mu;
}
inline std::map<TmaKey, CUtensorMap>& TmaCache() {
  static std::map<TmaKey, CUtensorMap> cache;
  return cache;
}

inline bool MakeTmaBf16(const void* base, int rows, int cols, int ld, int box_rows, CUtensorMap* out) {
  const TmaKey k{base, rows, cols, ld, box_rows};
  {
    std::lock_guard<std::mutex> g(TmaCacheMutex());
    auto it = TmaCache().find(k);
    if (it != TmaCache().end()) {
      *out = it->second;
      return true;
    }
  }
  EncodeTiledFn enc = GetEncodeTiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)kUmmaBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> g(TmaCacheMutex());
  TmaCache()[k] = m;
  *out = m;
  return true;
}

// Forgets the cached descriptors whose base address lies in [lo, hi) (memory that is being freed).
inline void ForgetTmaRange(const void* lo, const void* hi) {
  std::lock_guard<std::mutex> g(TmaCacheMutex());
  auto& c = TmaCache();
  for (auto it = c.begin(); it != c.end();) {
    if (it->first.p >= lo && it->first.p < hi) it = c.erase(it);
    else ++it;
  }
}

// ---- device: fused linear over a 128-row tile ---------------------------------------------------------

template <int NORM, class Epi, int BN>
__global__ void __launch_bounds__(kUmmaThreads, 1)
    LinearUmmaKernel(LinearArgs la, Epi epi, const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_w, int a_box_rows) {
  using L = UmmaSmem<BN>;
  constexpr int S = L::kStages;
  constexpr int kChunks = BN / 16;
  constexpr int kGroup = kChunks < 4 ? kChunks : 4;  // TMEM loads in flight before one wait (64 columns)
  constexpr bool kEarly = BN <= 32;  // epilogue reads issued before the main loop (registers allow it)
  const uint32_t stage_tx = (uint32_t)a_box_rows * kUmmaBK * 2 + (uint32_t)L::kB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * L::kStage);
  uint64_t* empty = full + S;
  uint64_t* final_bar = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_last = s_abort + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * kUmmaBM;
  // split-K: this CTA reduces k-blocks [kb0, kb0 + nk) of the row; gridDim.z CTAs share an output tile
  const int nk_all = CeilDiv(la.Kp, kUmmaBK);
  const int ks = gridDim.z, kz = blockIdx.z;
  const int kb0 = kz * nk_all / ks;
  const int nk = (kz + 1) * nk_all / ks - kb0;

  if (threadIdx.x == 0) {
    for (int st = 0; st < S; st++) {
      MbarInit(&full[st], 1);
      MbarInit(&empty[st], 1 + kUmmaThreads / 32);  // the MMA commit + one arrival per warp
    }
    MbarInit(final_bar, 1);
    *s_abort = 0;
    *s_last = 1;
    FenceMbarInit();
    PrefetchTmaDesc(&tmap_a);
    PrefetchTmaDesc(&tmap_w);
  }
  __syncwarp();
  if (warp == 0) {
    TmemAlloc(tmem_slot, L::kTmemCols);
    TmemRelinquish();
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  const uint32_t tmem = *tmem_slot;

  // Weights do not depend on earlier kernels: start their loads before waiting for the predecessor.
  if (threadIdx.x == 0) {
    for (int kb = 0; kb < nk && kb < S; kb++) {
      uint8_t* sa = smem + kb * L::kStage;
      MbarArriveExpectTx(&full[kb], stage_tx);
      TmaLoad2D(sa + L::kA, &tmap_w, &full[kb], (kb0 + kb) * kUmmaBK, n0);
    }
  }
  GridDepWait();
  GridDepLaunch();
  if (threadIdx.x == 0) {
    FenceProxyAsyncGlobal();
    for (int kb = 0; kb < nk && kb < S; kb++)
      TmaLoad2D(smem + kb * L::kStage, &tmap_a, &full[kb], (kb0 + kb) * kUmmaBK, m0);
  }
  const int r = warp * 32 + lane;
  const bool row_ok = m0 + r < la.M;
  const bool vec = epi.vec_ok(la.N);
  // the epilogue's global reads (residual, bias, RoPE table, KV page lookup) overlap the main loop
  typename Epi::Pre pre[kEarly ? kChunks : 1];
  if (kEarly && vec && row_ok) {
#pragma unroll
    for (int ch = 0; ch < (kEarly ? kChunks : 1); ch++)
      if (n0 + 16 * ch + 16 <= la.N) pre[ch] = epi.load16(m0 + r, n0 + 16 * ch);
  }

  // Main loop. Every thread waits for each stage and (for a norm) accumulates its own row's statistics
  // from the staged bf16 tile; thread 0 issues the MMAs of a stage and then refills the stage of the
  // previous iteration once its MMAs and the four warps are done with it, so the tensor pipe always has
  // the next stage's MMAs queued while thread 0 waits.
  float s1 = 0.f, s2 = 0.f;
  const uint32_t idesc = UmmaIdescBf16(kUmmaBM, BN);
  for (int kb = 0; kb < nk; kb++) {
    const int st = kb % S;
    const uint32_t ph = (kb / S) & 1;
    uint8_t* sa = smem + st * L::kStage;
    // warp-uniform outcome, so a lane never leaves the loop while its warp-mates wait in __syncwarp
    if (!__all_sync(0xffffffffu, MbarWaitBounded(&full[st], ph, kWaitLimit))) {
      if (lane == 0) atomicCAS(&g_shahd_device_error, 0, kDevErrUmmaTimeout);
      *s_abort = 1;
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
    if (lane == 0) MbarArrive(&empty[st]);
    if (threadIdx.x == 0) {
      TcgenFenceAfter();
      const uint64_t ad = SmemDescSw128(SmemAddr(sa));
      const uint64_t bd = SmemDescSw128(SmemAddr(sa + L::kA));
#pragma unroll
      for (int kk = 0; kk < kUmmaBK / 16; kk++)
        UmmaBf16(tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
      UmmaCommit(&empty[st]);
      const int kp = kb - 1;  // refill the previous iteration's stage with block kp + S
      if (kp >= 0 && kp + S < nk) {
        const int sp = kp % S;
        if (!MbarWaitBounded(&empty[sp], (kp / S) & 1, kWaitLimit)) {
          atomicCAS(&g_shahd_device_error, 0, kDevErrUmmaTimeout);
          *s_abort = 1;
        } else {
          uint8_t* sb = smem + sp * L::kStage;
          MbarArriveExpectTx(&full[sp], stage_tx);
          TmaLoad2D(sb, &tmap_a, &full[sp], (kb0 + kp + S) * kUmmaBK, m0);
          TmaLoad2D(sb + L::kA, &tmap_w, &full[sp], (kb0 + kp + S) * kUmmaBK, n0);
        }
      }
    }
  }
  if (threadIdx.x == 0 && !*s_abort) UmmaCommit(final_bar);
  float mu = 0.f, is = 1.f;
  if (NORM == kNormRms) {
    is = 1.0f / sqrtf(s2 / la.K + la.eps);
  } else if (NORM == kNormLayer) {
    mu = s1 / la.K;
    is = 1.0f / sqrtf(fmaxf(s2 / la.K - mu * mu, 0.f) + la.eps);
  }
  __syncthreads();
  if (!*s_abort && !MbarWaitBounded(final_bar, 0, kWaitLimit)) {
    if (lane == 0) atomicCAS(&g_shahd_device_error, 0, kDevErrUmmaTimeout);
    *s_abort = 1;
  }
  __syncthreads();
  TcgenFenceAfter();
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's 32 TMEM lanes
  // split-K within a cluster: each CTA leaves its partial tile in its own (now idle) stage memory; CTA
  // kz then sums rows [kz*128/ks, (kz+1)*128/ks) over the cluster in split order and runs their epilogue
  const bool kc = ks > 1 && la.kcluster != 0;
  float* spart = reinterpret_cast<float*>(smem);  // [kUmmaBM][BN]
  const bool own = !kc || r * ks / kUmmaBM == kz;
  if (kc) {
    if (!*s_abort) {
#pragma unroll
      for (int g = 0; g < kChunks; g += kGroup) {
        uint32_t u[kGroup][16];
#pragma unroll
        for (int q = 0; q < kGroup; q++) TmemLoad16(trow + (uint32_t)(16 * (g + q)), u[q]);
        TmemWaitLd();
#pragma unroll
        for (int q = 0; q < kGroup; q++)
#pragma unroll
          for (int i = 0; i < 4; i++)
            *reinterpret_cast<uint4*>(spart + (size_t)r * BN + 16 * (g + q) + 4 * i) =
                make_uint4(u[q][4 * i], u[q][4 * i + 1], u[q][4 * i + 2], u[q][4 * i + 3]);
      }
    }
    ClusterSync();  // every CTA of the cluster reaches both barriers, aborted or not
  } else if (!*s_abort && ks > 1) {
    // split-K: every CTA parks its partial tile in the workspace; the last CTA of the tile sums the
    // partials in split order (the result does not depend on which CTA finishes last) and runs the epilogue
    float* part = la.ws + ((size_t)(blockIdx.x * ks + kz) * kUmmaBM + r) * BN;
#pragma unroll
    for (int g = 0; g < kChunks; g += kGroup) {
      uint32_t u[kGroup][16];
#pragma unroll
      for (int q = 0; q < kGroup; q++) TmemLoad16(trow + (uint32_t)(16 * (g + q)), u[q]);
      TmemWaitLd();
      if (row_ok) {
#pragma unroll
        for (int q = 0; q < kGroup; q++) StoreNf<16>(part + 16 * (g + q), reinterpret_cast<const float*>(u[q]));
      }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_last = atomicAdd(la.ws_cnt + blockIdx.x, 1) == ks - 1;
    __syncthreads();
    if (*s_last) __threadfence();
  }
  if (!*s_abort && *s_last) {
    // Epilogue: thread = row (m0 + 32*warp + lane), 16 consecutive accumulator columns per chunk; the
    // TMEM loads of up to four chunks are in flight before one wait.
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int g = 0; g < kChunks; g += kGroup) {
      float vg[kGroup][16];
      if (kc) {
        if (row_ok && own) {
#pragma unroll
          for (int q = 0; q < kGroup; q++) {
#pragma unroll
            for (int j = 0; j < 16; j++) vg[q][j] = 0.f;
            for (int z = 0; z < ks; z++) {
#pragma unroll
              for (int i = 0; i < 4; i++) {
                const float4 t = LoadPeerF32x4(spart + (size_t)r * BN + 16 * (g + q) + 4 * i, (uint32_t)z);
                vg[q][4 * i] += t.x;
                vg[q][4 * i + 1] += t.y;
                vg[q][4 * i + 2] += t.z;
                vg[q][4 * i + 3] += t.w;
              }
            }
          }
        }
      } else if (ks > 1) {
        if (row_ok) {
#pragma unroll
          for (int q = 0; q < kGroup; q++) {
#pragma unroll
            for (int j = 0; j < 16; j++) vg[q][j] = 0.f;
            for (int z = 0; z < ks; z++) {
              const float4* src =
                  reinterpret_cast<const float4*>(la.ws + ((size_t)(blockIdx.x * ks + z) * kUmmaBM + r) * BN + 16 * (g + q));
#pragma unroll
              for (int i = 0; i < 4; i++) {
                const float4 t = __ldcg(src + i);
                vg[q][4 * i] += t.x;
                vg[q][4 * i + 1] += t.y;
                vg[q][4 * i + 2] += t.z;
                vg[q][4 * i + 3] += t.w;
              }
            }
          }
        }
      } else {
        uint32_t u[kGroup][16];
#pragma unroll
        for (int q = 0; q < kGroup; q++) TmemLoad16(trow + (uint32_t)(16 * (g + q)), u[q]);
        TmemWaitLd();
#pragma unroll
        for (int q = 0; q < kGroup; q++)
#pragma unroll
          for (int j = 0; j < 16; j++) vg[q][j] = __uint_as_float(u[q][j]);
      }
      if (!row_ok || !own) continue;
#pragma unroll
      for (int q = 0; q < kGroup; q++) {
        const int ch = g + q;
        const int nb = n0 + 16 * ch;
        float (&v)[16] = vg[q];
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
          if constexpr (kEarly) {
            epi.store16(m0 + r, nb, v, pre[ch]);
          } else {
            epi.store16(m0 + r, nb, v, epi.load16(m0 + r, nb));
          }
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
              epi.apply(m0 + r, n, v0, v1, la.N);
              if constexpr (IsLogits<Epi>::value) {
                ArgmaxMerge(bv, bi, v0, n);
                if (n + 1 < la.N) ArgmaxMerge(bv, bi, v1, n + 1);
              }
            }
          }
        }
      }
    }
    if constexpr (IsLogits<Epi>::value) {
      if (row_ok) {
        la.am_val[(size_t)(m0 + r) * gridDim.x + blockIdx.x] = bv;
        la.am_idx[(size_t)(m0 + r) * gridDim.x + blockIdx.x] = bi;
      }
    }
    if (ks > 1 && !kc && threadIdx.x == 0) la.ws_cnt[blockIdx.x] = 0;  // ready for the next launch
  }
  if (kc) ClusterSync();  // the peers are done reading this CTA's partial tile
  TcgenFenceBefore();
  __syncthreads();
  __syncwarp();
  if (warp == 0) TmemDealloc(tmem, L::kTmemCols);
}

template <int NORM, class Epi, int BN>
void LaunchUmmaLinearBN(const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  CUtensorMap tw, ta;
  const int box = UmmaBoxRows(la.M);
  if (!MakeTmaBf16(la.w, la.N, la.Kp, la.Kp, BN, &tw) || !MakeTmaBf16(la.ab, la.a_rows, la.Kp, la.ldab, box, &ta)) {
    NoteLaunchError(cudaErrorInvalidValue, "cuTensorMapEncodeTiled for a projection");  // reported by the caller
    return;
  }
  if (!EnsureKernelAttrs((const void*)LinearUmmaKernel<NORM, Epi, BN>, UmmaSmem<BN>::kBytes)) return;
  const int ks = (NORM == kNormNone && la.ws != nullptr) ? UmmaKSplit(la.M, la.N, la.Kp) : 1;
  dim3 grid(CeilDiv(la.N, BN), CeilDiv(la.M, kUmmaBM), ks);
  static_assert(UmmaSmem<BN>::kStages * UmmaSmem<BN>::kStage >= kUmmaBM * BN * 4, "partial tile fits the stages");
  if (ks > 1) {  // the split CTAs of a tile reduce through distributed shared memory
    LinearArgs lc = la;
    lc.kcluster = 1;
    LaunchPdlCluster(LinearUmmaKernel<NORM, Epi, BN>, grid, dim3(kUmmaThreads), UmmaSmem<BN>::kBytes, dim3(1, 1, ks), st,
                     lc, epi, ta, tw, box);
  } else {
    LaunchPdl(LinearUmmaKernel<NORM, Epi, BN>, grid, dim3(kUmmaThreads), UmmaSmem<BN>::kBytes, st, la, epi, ta, tw,
              box);
  }
}

template <int NORM, class Epi>
void LaunchUmmaLinear(const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  const int bn = UmmaBN(la.M, la.N);
  if (bn == 16) LaunchUmmaLinearBN<NORM, Epi, 16>(la, epi, st);
  else if (bn == 32) LaunchUmmaLinearBN<NORM, Epi, 32>(la, epi, st);
  else if (bn == 64) LaunchUmmaLinearBN<NORM, Epi, 64>(la, epi, st);
  else LaunchUmmaLinearBN<NORM, Epi, 128>(la, epi, st);
}

}  // namespace shahd
