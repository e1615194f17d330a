// Persistent warp-specialized tcgen05 GEMM with fused epilogues: the batched-prefill projections
// (MatMulRow over many rows, CachedRowMath.ts:14-23, with the norm of NormRow, :25-56, and the epilogues of
// the decode chain: RoPE + KV append, residual, SwiGLU/GeGLU, ReLU) and the device-pointer MatMulNT
// (MatMulNT.ts:27-43) share it.
//
// One CTA per SM loops over 128-row x BN-column output tiles (row-block major, so consecutive tiles of the
// grid share the activation rows in L2):
//   warp 0 (one thread): TMA loads of the activation tile [128 x 64] and the weight tile [BN x 64] per
//     k-block into a ring of stages (128-byte swizzle, K-major);
//   warp 1 (one thread): tcgen05.mma kind::f16 (M 128, N BN, K 16) into one of two TMEM accumulators, so the
//     next tile's MMAs run while the epilogue drains the previous one;
//   warps 2..: the epilogue, two or four warps per TMEM lane quadrant (32 rows), each on a part of the
//     tile's columns: tcgen05.ld of 16-column chunks, the row's norm statistics (precomputed by RowStatsKernel from
//     the fp32 residual), the fused epilogue functor; the epilogue's global reads (residual, RoPE rows, KV
//     page lookups) are issued before the accumulator is waited for.
// Every mbarrier wait is bounded; on timeout the kernel records an error, stops issuing work, frees its
// TMEM and returns.
#pragma once

#include <type_traits>

#include "umma_linear.cuh"

namespace shahd {

template <int BN>
struct PersistCfg {
  static constexpr int kStageBytes = (kUmmaBM + BN) * kUmmaBK * 2;  // 32 KB (BN 128), 48 KB (BN 256)
  static constexpr int kStages = BN >= 256 ? 4 : 6;
  static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 512 /*barriers*/;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
};
// Epilogue warps: sixteen for epilogues that read nothing before the accumulator (the gated MLP, whose
// activation math is the longest part of a tile), eight for those whose early reads hold registers.
template <class Epi>
struct PersistEpi {
  static constexpr int kWarps = sizeof(typename Epi::Pre) <= 1 ? 16 : 8;
  static constexpr int kThreads = 64 + 32 * kWarps;
  static constexpr int kColParts = kWarps / 4;  // epilogue warps per TMEM lane quadrant (column parts)
};

// fp32 output rows (MatMulNT: out = A.B^T, or out += A.B^T when acc)
struct EpiF32Out {
  float* out;
  int ldo;
  int acc;
  __device__ __forceinline__ void apply(int m, int n, float v0, float v1, int N) const {
    float* o = out + (size_t)m * ldo + n;
    o[0] = acc ? o[0] + v0 : v0;
    if (n + 1 < N) o[1] = acc ? o[1] + v1 : v1;
  }
  struct Pre {
    float o[16];
  };
  __device__ __forceinline__ bool vec_ok(int N) const { return ldo % 4 == 0; }
  __device__ __forceinline__ Pre load16(int m, int n) const {
    Pre pr;
    if (acc) Load16f(out + (size_t)m * ldo + n, pr.o);
    return pr;
  }
  __device__ __forceinline__ void store16(int m, int n, float (&v)[16], const Pre& pr) const {
    if (acc) {
#pragma unroll
      for (int i = 0; i < 16; i++) v[i] += pr.o[i];
    }
    StoreNf<16>(out + (size_t)m * ldo + n, v);
  }
};

// Per-row norm statistics of the fp32 residual rows x[0 .. M): stats[2r] = mean (LayerNorm; 0 for RMSNorm),
// stats[2r + 1] = 1 / sqrt(variance (or mean square) + eps). One warp per row.
__global__ void __launch_bounds__(256) RowStatsKernel(const float* x, int ldx, int K, int M, int norm, float eps,
                                                      float* stats) {
  GridDepWait();
  GridDepLaunch();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const float* xr = x + (size_t)row * ldx;
  float s = 0.f;
  for (int k = lane; k < K; k += 32) s += xr[k];
  const float mu = norm == kNormLayer ? WarpSum(s) / K : 0.f;
  float v = 0.f;
  for (int k = lane; k < K; k += 32) {
    const float d = xr[k] - mu;
    v += d * d;
  }
  v = WarpSum(v);
  if (lane == 0) {
    stats[2 * row] = mu;
    stats[2 * row + 1] = 1.0f / sqrtf(v / K + eps);
  }
}

template <int NORM, class Epi, int BN>
__global__ void __launch_bounds__(PersistEpi<Epi>::kThreads, 1)
    LinearPersistKernel(LinearArgs la, Epi epi, const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_w) {
  using P = PersistCfg<BN>;
  constexpr int S = P::kStages;
  constexpr int kEpiWarps = PersistEpi<Epi>::kWarps;
  constexpr int kColsW = BN / PersistEpi<Epi>::kColParts;  // columns of the tile per epilogue warp
  constexpr int kChunksW = kColsW / 16;          // 16-column chunks per epilogue warp
  // chunks whose epilogue reads are in flight together: fewer when they hold many registers
  constexpr int kGroupW = (NORM == kNormLayer || sizeof(typename Epi::Pre) > 64) ? 2 : 4;
  constexpr int kGroup = kGroupW < kChunksW ? kGroupW : kChunksW;
  static_assert(kChunksW % kGroup == 0, "whole groups per warp");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * P::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;  // [2]
  uint64_t* tempty = tfull + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = CeilDiv(la.N, BN), tiles = tiles_n * CeilDiv(la.M, kUmmaBM);
  const int nk = CeilDiv(la.Kp, kUmmaBK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      MbarInit(&full[s], 1);
      MbarInit(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      MbarInit(&tfull[b], 1);
      MbarInit(&tempty[b], kEpiWarps);
    }
    *s_abort = 0;
    FenceMbarInit();
    PrefetchTmaDesc(&tmap_a);
    PrefetchTmaDesc(&tmap_w);
  }
  __syncwarp();
  if (warp == 1) {
    TmemAlloc(tmem_slot, P::kTmemCols);
    TmemRelinquish();
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  const uint32_t tmem = *tmem_slot;
  GridDepWait();  // the activation rows and the norm statistics come from the preceding launches
  GridDepLaunch();

  if (warp == 0) {
    if (lane == 0) {
      FenceProxyAsyncGlobal();
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !*s_abort; t += gridDim.x) {
        const int m0 = (t / tiles_n) * kUmmaBM, n0 = (t % tiles_n) * BN;
        for (int kb = 0; kb < nk; kb++, it++) {
          const int s = it % S;
          if (!MbarWaitBounded(&empty[s], ((it / S) & 1) ^ 1, kWaitLimit)) {
            atomicCAS(&g_shahd_device_error, 0, kDevErrGemmTimeout);
            *s_abort = 1;
            break;
          }
          uint8_t* sa = smem + s * P::kStageBytes;
          MbarArriveExpectTx(&full[s], P::kStageBytes);
          TmaLoad2D(sa, &tmap_a, &full[s], kb * kUmmaBK, m0);
          TmaLoad2D(sa + kUmmaBM * kUmmaBK * 2, &tmap_w, &full[s], kb * kUmmaBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = UmmaIdescBf16(kUmmaBM, BN);
      int it = 0, tc = 0;
      for (int t = blockIdx.x; t < tiles && !*s_abort; t += gridDim.x, tc++) {
        const int buf = tc & 1;
        if (!MbarWaitBounded(&tempty[buf], ((tc >> 1) & 1) ^ 1, kWaitLimit)) {
          atomicCAS(&g_shahd_device_error, 0, kDevErrGemmTimeout);
          *s_abort = 1;
          break;
        }
        TcgenFenceAfter();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < nk; kb++, it++) {
          const int s = it % S;
          if (!MbarWaitBounded(&full[s], (it / S) & 1, kWaitLimit)) {
            atomicCAS(&g_shahd_device_error, 0, kDevErrGemmTimeout);
            *s_abort = 1;
            break;
          }
          TcgenFenceAfter();
          uint8_t* sa = smem + s * P::kStageBytes;
          const uint64_t ad = SmemDescSw128(SmemAddr(sa));
          const uint64_t bd = SmemDescSw128(SmemAddr(sa + kUmmaBM * kUmmaBK * 2));
#pragma unroll
          for (int kk = 0; kk < kUmmaBK / 16; kk++)
            UmmaBf16(d, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          UmmaCommit(&empty[s]);
        }
        if (*s_abort) break;
        UmmaCommit(&tfull[buf]);
      }
    }
  } else {
    // epilogue: warps 2.., TMEM lane quadrant warp % 4, column part (warp - 2) / 4
    const int quad = warp & 3, part = (warp - 2) >> 2;
    const bool vec = epi.vec_ok(la.N);
    int tc = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, tc++) {
      const int buf = tc & 1;
      const int m0 = (t / tiles_n) * kUmmaBM, n0 = (t % tiles_n) * BN + part * kColsW;
      const int row = m0 + quad * 32 + lane;
      const bool row_ok = row < la.M;
      float mu = 0.f, is = 1.f;
      if (NORM != kNormNone && row_ok) {
        mu = __ldg(la.stats + 2 * row);
        is = __ldg(la.stats + 2 * row + 1);
      }
      typename Epi::Pre pre[kGroup];
      auto issue_pre = [&](int g) {
        if (!vec || !row_ok) return;
#pragma unroll
        for (int q = 0; q < kGroup; q++)
          if (n0 + 16 * (g + q) + 16 <= la.N) pre[q] = epi.load16(row, n0 + 16 * (g + q));
      };
      issue_pre(0);  // global reads in flight while the accumulator is finished
      if (!MbarWaitBounded(&tfull[buf], (tc >> 1) & 1, kWaitLimit)) {
        if (lane == 0) atomicCAS(&g_shahd_device_error, 0, kDevErrGemmTimeout);
        *s_abort = 1;
        break;
      }
      TcgenFenceAfter();
      const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN + part * kColsW);
#pragma unroll
      for (int g = 0; g < kChunksW; g += kGroup) {
        uint32_t u[kGroup][16];
#pragma unroll
        for (int q = 0; q < kGroup; q++) TmemLoad16(trow + (uint32_t)(16 * (g + q)), u[q]);
        TmemWaitLd();
        if (row_ok) {
#pragma unroll
          for (int q = 0; q < kGroup; q++) {
            const int nb = n0 + 16 * (g + q);
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] = __uint_as_float(u[q][j]);
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
              epi.store16(row, nb, v, pre[q]);
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
                  epi.apply(row, n, v0, v1, la.N);
                }
              }
            }
          }
        }
        if (g + kGroup < kChunksW) issue_pre(g + kGroup);
      }
      TcgenFenceBefore();
      __syncwarp();
      if (lane == 0) MbarArrive(&tempty[buf]);
    }
  }
  TcgenFenceBefore();
  __syncthreads();
  __syncwarp();
  if (warp == 1) TmemDealloc(tmem, P::kTmemCols);
}

extern int g_persist_linear;

inline int NumSmsOfCurrentDevice() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (!cache[dev & 63]) cudaDeviceGetAttribute(&cache[dev & 63], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev & 63] > 0 ? cache[dev & 63] : 148;
}

// The (norm, epilogue) pairs the batched prefill runs through the persistent kernel: the norm-consuming
// projections (QKV + RoPE + KV append, MLP up) and the residual ones (O, MLP down). The LM head keeps the
// per-CTA argmax partials of LinearUmmaKernel.
template <int NORM, class Epi>
struct PersistUsed {
  static constexpr bool value = NORM == kNormNone ? std::is_same<Epi, EpiResid>::value
                                                  : (std::is_same<Epi, EpiQKV>::value || std::is_same<Epi, EpiGated>::value ||
                                                     std::is_same<Epi, EpiReluFc>::value);
};

// Launches the persistent kernel over every SM (or fewer CTAs than tiles); returns false (the launch error
// recorded) when a TMA map cannot be encoded or the kernel's attributes cannot be set.
template <int NORM, class Epi, int BN>
bool LaunchPersistLinearBN(const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  CUtensorMap ta, tw;
  if (!MakeTmaBf16(la.ab, la.a_rows, la.Kp, la.ldab, kUmmaBM, &ta) || !MakeTmaBf16(la.w, la.N, la.Kp, la.Kp, BN, &tw)) {
    NoteLaunchError(cudaErrorInvalidValue, "cuTensorMapEncodeTiled for a persistent projection");
    return false;
  }
  if (!EnsureKernelAttrs((const void*)LinearPersistKernel<NORM, Epi, BN>, PersistCfg<BN>::kSmem)) return false;
  const int tiles = CeilDiv(la.N, BN) * CeilDiv(la.M, kUmmaBM);
  const int grid = std::min(tiles, NumSmsOfCurrentDevice());
  LaunchPdl(LinearPersistKernel<NORM, Epi, BN>, dim3(grid), dim3(PersistEpi<Epi>::kThreads), PersistCfg<BN>::kSmem, st,
            la, epi, ta, tw);
  return true;
}

// Column tile: 256 when the wide tiles still give every SM work, 128 otherwise.
inline int PersistBN(int M, int N, int num_sms) {
  return CeilDiv(N, 256) * CeilDiv(M, kUmmaBM) >= num_sms ? 256 : 128;
}

template <int NORM, class Epi>
bool LaunchPersistLinear(const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  if (PersistBN(la.M, la.N, NumSmsOfCurrentDevice()) == 256) return LaunchPersistLinearBN<NORM, Epi, 256>(la, epi, st);
  return LaunchPersistLinearBN<NORM, Epi, 128>(la, epi, st);
}

}  // namespace shahd
