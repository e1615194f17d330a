// Tensor-core (tcgen05 / TMEM / TMA) kernels for sm_100a.
//
// LinearUmmaKernel: the batched-rows regime of every decode/prefill projection. 128-row x BN-column
// output tile per CTA; the weight tile [BN x 64] arrives by TMA (128-byte swizzle); the activation
// tile [128 x 64] is produced by the CTA's own threads from fp32 rows with the layer norm applied
// (NormRow, CachedRowMath.ts:25-56) and converted to bf16 into the same swizzled K-major layout; one
// thread issues tcgen05.mma (M=128, N=BN, K=16) into a TMEM accumulator; the four warps read their
// 32-lane quadrant back with tcgen05.ld and run the fused epilogue (RoPE + KV append, residual add,
// SwiGLU/GeGLU, LM head + argmax).
//
// GemmNtBf16Kernel: out[M,N] (+)= A[M,K] · B[N,K]ᵀ with both operands bf16 in global memory, both
// fed by TMA, warp-specialized (producer warp, MMA warp, 4 epilogue warps) — the MatMulNT operator.
//
// Every mbarrier wait is bounded; on timeout the kernel records an error code in g_shahd_device_error,
// skips the remaining work, releases its TMEM and returns.
#pragma once

#include <map>
#include <mutex>

#include "common.cuh"
#include "decode_kernels.cuh"

namespace shahd {

constexpr uint32_t kWaitLimit = 1u << 22;

constexpr int kUmmaBM = 128;
constexpr int kUmmaBK = 64;
constexpr int kUmmaStages = 4;
constexpr int kUmmaThreads = 128;

// Rows at which a projection switches from the SIMT (CUDA-core) kernel to tensor-core tiles. Settable
// through ShahdSetTensorCoreMinRows / SetScalarKernels (test hooks, process-wide).
extern int g_umma_min_rows;
#define kUmmaMinRows (::shahd::g_umma_min_rows)

__host__ inline int UmmaBN(int M, int N) {
  if (M > kUmmaBM) return 128;
  return N <= 1024 ? 32 : 64;
}
__host__ inline int UmmaGridN(int N) { return CeilDiv(N, 32); }  // upper bound of N tiles (BN >= 32)

inline bool UmmaLinearSupported(const LinearArgs& la) { return la.Kp % 8 == 0 && la.N >= 1; }

template <int BN>
struct UmmaSmem {
  static constexpr int kA = kUmmaBM * kUmmaBK * 2;  // 16 KB
  static constexpr int kB = BN * kUmmaBK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kBytes = kUmmaStages * kStage + 1024 /*align*/ + 256 /*barriers*/ + 2 * kUmmaBM * 4;
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

// Cached per (pointer, shape, box): weights are fixed for a session's lifetime.
inline bool MakeTmaBf16(const void* base, int rows, int cols, int ld, int box_rows, CUtensorMap* out) {
  struct Key {
    const void* p;
    int r, c, ld, b;
    bool operator<(const Key& o) const {
      if (p != o.p) return p < o.p;
      if (r != o.r) return r < o.r;
      if (c != o.c) return c < o.c;
      if (ld != o.ld) return ld < o.ld;
      return b < o.b;
    }
  };
  static std::mutex mu;
  static std::map<Key, CUtensorMap> cache;
  Key k{base, rows, cols, ld, box_rows};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(k);
    if (it != cache.end()) {
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
  std::lock_guard<std::mutex> g(mu);
  cache[k] = m;
  *out = m;
  return true;
}

// Forget cached descriptors that point into [lo, hi) (a session freeing its weights).
inline void ForgetTmaRange(const void* lo, const void* hi) { (void)lo; (void)hi; }

// ---- device: fused linear over a 128-row tile ---------------------------------------------------------

template <int NORM, class Epi, int BN>
__global__ void __launch_bounds__(kUmmaThreads, 1)
    LinearUmmaKernel(LinearArgs la, Epi epi, const __grid_constant__ CUtensorMap tmap_w) {
  using L = UmmaSmem<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_b = reinterpret_cast<uint64_t*>(smem + kUmmaStages * L::kStage);
  uint64_t* mma_done = full_b + kUmmaStages;
  uint64_t* final_bar = mma_done + kUmmaStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);
  float* s_mu = reinterpret_cast<float*>(smem + kUmmaStages * L::kStage + 256);
  float* s_is = s_mu + kUmmaBM;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * kUmmaBM;
  const int rows = min(kUmmaBM, la.M - m0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kUmmaStages; s++) {
      MbarInit(&full_b[s], 1);
      MbarInit(&mma_done[s], 1);
    }
    MbarInit(final_bar, 1);
    *s_abort = 0;
    FenceMbarInit();
    PrefetchTmaDesc(&tmap_w);
  }
  __syncwarp();
  if (warp == 0) {
    TmemAlloc(tmem_slot, BN);
    TmemRelinquish();
  }
  // Row statistics of the norm (one warp per 32 rows).
  if (NORM != kNormNone) {
    for (int r = warp * 32; r < warp * 32 + 32; r++) {
      if (r >= rows) break;
      const float* src = la.a + (size_t)(m0 + r) * la.lda;
      float mu = 0.f, is;
      if (NORM == kNormRms) {
        float ss = 0.f;
        for (int k = lane; k < la.K; k += 32) ss += src[k] * src[k];
        ss = WarpSum(ss);
        is = 1.0f / sqrtf(ss / la.K + la.eps);
      } else {
        float s = 0.f;
        for (int k = lane; k < la.K; k += 32) s += src[k];
        mu = WarpSum(s) / la.K;
        float v = 0.f;
        for (int k = lane; k < la.K; k += 32) {
          float t = src[k] - mu;
          v += t * t;
        }
        v = WarpSum(v) / la.K;
        is = 1.0f / sqrtf(v + la.eps);
      }
      if (lane == 0) {
        s_mu[r] = mu;
        s_is[r] = is;
      }
    }
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  const uint32_t tmem = *tmem_slot;
  const uint32_t idesc = UmmaIdescBf16(kUmmaBM, BN);
  const int nk = CeilDiv(la.Kp, kUmmaBK);

  for (int kb = 0; kb < nk; kb++) {
    const int st = kb % kUmmaStages;
    uint8_t* sa = smem + st * L::kStage;
    uint8_t* sb = sa + L::kA;
    if (kb >= kUmmaStages) {
      // the MMAs that read this stage kUmmaStages iterations ago must be done before it is refilled
      if (!MbarWaitBounded(&mma_done[st], ((kb / kUmmaStages) - 1) & 1, kWaitLimit)) {
        if (lane == 0) atomicCAS(&g_shahd_device_error, 0, kDevErrUmmaTimeout);
        *s_abort = 1;
      }
    }
    __syncthreads();
    if (*s_abort) break;
    if (threadIdx.x == 0) {
      MbarArriveExpectTx(&full_b[st], L::kB);
      TmaLoad2D(sb, &tmap_w, &full_b[st], kb * kUmmaBK, n0);
    }
    // A tile: 128 rows x 64 k, fp32 -> (norm) -> bf16, two rows per warp instruction (16 lanes x 4 k).
    const int k0 = kb * kUmmaBK;
    const int half = lane >> 4, kl = (lane & 15) * 4;
    for (int rr = warp * 32; rr < warp * 32 + 32; rr += 2) {
      const int r = rr + half;
      const int k = k0 + kl;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (r < rows) {
        const float* src = la.a + (size_t)(m0 + r) * la.lda;
        if (k + 3 < la.K && (la.lda & 3) == 0) {
          const float4 t = *reinterpret_cast<const float4*>(src + k);
          v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; j++)
            if (k + j < la.K) v[j] = src[k + j];
        }
        if (NORM != kNormNone) {
          const float mu = s_mu[r], is = s_is[r];
#pragma unroll
          for (int j = 0; j < 4; j++) {
            if (k + j < la.K) {
              if (NORM == kNormRms) v[j] = la.gamma[k + j] * v[j] * is;
              else v[j] = la.gamma[k + j] * ((v[j] - mu) * is) + la.beta[k + j];
            }
          }
        }
      }
      __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]);
      __nv_bfloat162 p1 = __floats2bfloat162_rn(v[2], v[3]);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&p0);
      pk.y = *reinterpret_cast<uint32_t*>(&p1);
      const int chunk = kl >> 3, sub = (kl & 7) * 2;  // 16-byte chunk and byte offset inside it
      *reinterpret_cast<uint2*>(sa + Sw128Offset(r, chunk) + sub) = pk;
    }
    FenceProxyAsyncShared();
    __syncthreads();
    if (threadIdx.x == 0) {
      if (!MbarWaitBounded(&full_b[st], (kb / kUmmaStages) & 1, kWaitLimit)) {
        atomicCAS(&g_shahd_device_error, 0, kDevErrUmmaTimeout);
        *s_abort = 1;
      } else {
        TcgenFenceAfter();
        const uint64_t ad = SmemDescSw128(SmemAddr(sa));
        const uint64_t bd = SmemDescSw128(SmemAddr(sb));
#pragma unroll
        for (int kk = 0; kk < kUmmaBK / 16; kk++)
          UmmaBf16(tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        UmmaCommit(&mma_done[st]);
      }
    }
  }
  __syncthreads();
  const bool ok = *s_abort == 0;
  if (ok && threadIdx.x == 0) UmmaCommit(final_bar);
  if (ok && !MbarWaitBounded(final_bar, 0, kWaitLimit)) {
    if (lane == 0) atomicCAS(&g_shahd_device_error, 0, kDevErrUmmaTimeout);
    *s_abort = 1;
  }
  __syncthreads();
  TcgenFenceAfter();
  if (*s_abort == 0) {
    // Epilogue: thread = row (m0 + 32*warp + lane), 16 consecutive accumulator columns per TMEM load.
    const int r = warp * 32 + lane;
    const bool row_ok = r < rows;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      uint32_t u[16];
      TmemLoad16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, u);
      TmemWaitLd();
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const int n = n0 + c + j;
          if (n < la.N) {
            float v0 = __uint_as_float(u[j]), v1 = __uint_as_float(u[j + 1]);
            epi.apply(m0 + r, n, v0, v1, la.N);
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
        la.am_val[(size_t)(m0 + r) * gridDim.x + blockIdx.x] = bv;
        la.am_idx[(size_t)(m0 + r) * gridDim.x + blockIdx.x] = bi;
      }
    }
  }
  TcgenFenceBefore();
  __syncthreads();
  __syncwarp();
  if (warp == 0) TmemDealloc(tmem, BN);
}

template <int NORM, class Epi, int BN>
void LaunchUmmaLinearBN(const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  CUtensorMap tm;
  if (!MakeTmaBf16(la.w, la.N, la.Kp, la.Kp, BN, &tm)) return;  // launch error surfaces via CheckLaunch
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(LinearUmmaKernel<NORM, Epi, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         UmmaSmem<BN>::kBytes);
    configured = true;
  }
  dim3 grid(CeilDiv(la.N, BN), CeilDiv(la.M, kUmmaBM));
  LinearUmmaKernel<NORM, Epi, BN><<<grid, kUmmaThreads, UmmaSmem<BN>::kBytes, st>>>(la, epi, tm);
}

template <int NORM, class Epi>
void LaunchUmmaLinear(const LinearArgs& la, const Epi& epi, cudaStream_t st) {
  const int bn = UmmaBN(la.M, la.N);
  if (bn == 32) LaunchUmmaLinearBN<NORM, Epi, 32>(la, epi, st);
  else if (bn == 64) LaunchUmmaLinearBN<NORM, Epi, 64>(la, epi, st);
  else LaunchUmmaLinearBN<NORM, Epi, 128>(la, epi, st);
}

}  // namespace shahd
