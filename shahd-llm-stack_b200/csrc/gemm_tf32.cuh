// fp32 MatMulNT on the tensor cores (tcgen05.mma kind::tf32) with fp32-level accuracy.
//
// The reference's f32 seam (MatMulNTF32 / MatMulF32, GoKernels/ffi/matmul.go:329-357) accumulates fp32
// products; a backend must agree with it to 1e-4 (Tests/Compute.Test.ts:109-145). One TF32 pass (10-bit
// mantissa inputs) misses that at K ~ 1024, so each operand is split once into two TF32-representable parts,
// x = hi + lo with hi = tf32(x) and lo = tf32(x - hi), and every k-block issues three MMAs into the same fp32
// TMEM accumulator: lo_a·hi_b + hi_a·lo_b + hi_a·hi_b (the lo·lo term is below fp32 rounding). Operands are
// K-major fp32 rows loaded by TMA (32 elements = one 128-byte swizzle row per k-block); the kernel is
// persistent and warp-specialized like the bf16 GEMM: warp 0 issues TMA, warp 1 issues MMAs into one of two
// TMEM accumulators, warps 2-5 drain the other one.
#pragma once

#include "common.cuh"
#include "decode_kernels.cuh"
#include "umma_linear.cuh"

namespace shahd {

constexpr int kT32BM = 128, kT32BN = 128, kT32BK = 32;  // kT32BK fp32 = one 128-byte row
constexpr int kT32Stages = 3;
constexpr int kT32Tile = 128 * kT32BK * 4;     // one operand tile: 128 rows x 32 fp32 = 16 KB
constexpr int kT32StageBytes = 4 * kT32Tile;   // A hi, A lo, B hi, B lo
constexpr int kT32Smem = kT32Stages * kT32StageBytes + 1024 + 256;
constexpr int kT32Threads = 192;
constexpr int kDevErrTf32Timeout = 6;

// Instruction descriptor, kind::tf32: TF32 A/B (format 2), fp32 D, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t UmmaIdescTf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void UmmaTf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ float RoundTf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi = tf32(x), lo = tf32(x - hi), element by element (both stay fp32 words the MMA reads as TF32).
__global__ void SplitTf32Kernel(const float* x, float* hi, float* __restrict__ lo, size_t n) {  // hi may be x
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float h = RoundTf32(v);
    hi[i] = h;
    lo[i] = RoundTf32(v - h);
  }
}

// out[M,N] (+)= A[M,K] · B[N,K]ᵀ from the split operands (tensor maps of A hi/lo and B hi/lo).
__global__ void __launch_bounds__(kT32Threads, 1)
    GemmNtTf32x3Kernel(const __grid_constant__ CUtensorMap tah, const __grid_constant__ CUtensorMap tal,
                       const __grid_constant__ CUtensorMap tbh, const __grid_constant__ CUtensorMap tbl, float* out, int M,
                       int N, int K, int acc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kT32Stages * kT32StageBytes);
  uint64_t* empty = full + kT32Stages;
  uint64_t* tfull = empty + kT32Stages;  // [2]
  uint64_t* tempty = tfull + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = CeilDiv(N, kT32BN), tiles = tiles_n * CeilDiv(M, kT32BM);
  const int nk = CeilDiv(K, kT32BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kT32Stages; s++) {
      MbarInit(&full[s], 1);
      MbarInit(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      MbarInit(&tfull[b], 1);
      MbarInit(&tempty[b], 4);
    }
    *s_abort = 0;
    FenceMbarInit();
    PrefetchTmaDesc(&tah);
    PrefetchTmaDesc(&tal);
    PrefetchTmaDesc(&tbh);
    PrefetchTmaDesc(&tbl);
  }
  __syncwarp();
  if (warp == 1) {
    TmemAlloc(tmem_slot, 2 * kT32BN);
    TmemRelinquish();
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !*s_abort; t += gridDim.x) {
        const int m0 = (t / tiles_n) * kT32BM, n0 = (t % tiles_n) * kT32BN;
        for (int kb = 0; kb < nk; kb++, it++) {
          const int s = it % kT32Stages;
          if (!MbarWaitBounded(&empty[s], ((it / kT32Stages) & 1) ^ 1, kWaitLimit)) {
            atomicCAS(&g_shahd_device_error, 0, kDevErrTf32Timeout);
            *s_abort = 1;
            break;
          }
          uint8_t* sa = smem + s * kT32StageBytes;
          MbarArriveExpectTx(&full[s], kT32StageBytes);
          TmaLoad2D(sa, &tah, &full[s], kb * kT32BK, m0);
          TmaLoad2D(sa + kT32Tile, &tal, &full[s], kb * kT32BK, m0);
          TmaLoad2D(sa + 2 * kT32Tile, &tbh, &full[s], kb * kT32BK, n0);
          TmaLoad2D(sa + 3 * kT32Tile, &tbl, &full[s], kb * kT32BK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = UmmaIdescTf32(kT32BM, kT32BN);
      int it = 0, tc = 0;
      for (int t = blockIdx.x; t < tiles && !*s_abort; t += gridDim.x, tc++) {
        const int buf = tc & 1;
        if (!MbarWaitBounded(&tempty[buf], ((tc >> 1) & 1) ^ 1, kWaitLimit)) {
          atomicCAS(&g_shahd_device_error, 0, kDevErrTf32Timeout);
          *s_abort = 1;
          break;
        }
        TcgenFenceAfter();
        const uint32_t d = tmem + (uint32_t)(buf * kT32BN);
        for (int kb = 0; kb < nk; kb++, it++) {
          const int s = it % kT32Stages;
          if (!MbarWaitBounded(&full[s], (it / kT32Stages) & 1, kWaitLimit)) {
            atomicCAS(&g_shahd_device_error, 0, kDevErrTf32Timeout);
            *s_abort = 1;
            break;
          }
          TcgenFenceAfter();
          uint8_t* sa = smem + s * kT32StageBytes;
          const uint64_t ah = SmemDescSw128(SmemAddr(sa)), al = SmemDescSw128(SmemAddr(sa + kT32Tile));
          const uint64_t bh = SmemDescSw128(SmemAddr(sa + 2 * kT32Tile)), bl = SmemDescSw128(SmemAddr(sa + 3 * kT32Tile));
#pragma unroll
          for (int kk = 0; kk < kT32BK / 8; kk++) {  // K = 8 TF32 (32 bytes) per MMA
            const uint64_t o = (uint64_t)(kk * 2);
            UmmaTf32(d, al + o, bh + o, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            UmmaTf32(d, ah + o, bl + o, idesc, 1u);
            UmmaTf32(d, ah + o, bh + o, idesc, 1u);
          }
          UmmaCommit(&empty[s]);
        }
        if (*s_abort) break;
        UmmaCommit(&tfull[buf]);
      }
    }
  } else {
    // epilogue warps 2..5 own TMEM lane quadrants (warp % 4)
    const int quad = warp & 3;
    int tc = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, tc++) {
      const int buf = tc & 1;
      if (!MbarWaitBounded(&tfull[buf], (tc >> 1) & 1, kWaitLimit)) {
        if (lane == 0) atomicCAS(&g_shahd_device_error, 0, kDevErrTf32Timeout);
        *s_abort = 1;
        break;
      }
      TcgenFenceAfter();
      const int m0 = (t / tiles_n) * kT32BM, n0 = (t % tiles_n) * kT32BN;
      const int row = m0 + quad * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < kT32BN; c += 16) {
        uint32_t u[16];
        TmemLoad16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * kT32BN + c), u);
        TmemWaitLd();
        if (row < M) {
          float* o = out + (size_t)row * N + n0 + c;
          if (n0 + c + 16 <= N && (N & 3) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
              float4 v = make_float4(__uint_as_float(u[j]), __uint_as_float(u[j + 1]), __uint_as_float(u[j + 2]),
                                     __uint_as_float(u[j + 3]));
              if (acc) {
                const float4 p = *reinterpret_cast<const float4*>(o + j);
                v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
              }
              *reinterpret_cast<float4*>(o + j) = v;
            }
          } else {
            for (int j = 0; j < 16; j++)
              if (n0 + c + j < N) o[j] = acc ? o[j] + __uint_as_float(u[j]) : __uint_as_float(u[j]);
          }
        }
      }
      TcgenFenceBefore();
      __syncwarp();
      if (lane == 0) MbarArrive(&tempty[buf]);
    }
  }
  TcgenFenceBefore();
  __syncthreads();
  __syncwarp();
  if (warp == 1) TmemDealloc(tmem, 2 * kT32BN);
}

// TMA descriptor of an fp32 row-major [rows, cols] matrix, box [128 rows x 32 columns], 128-byte swizzle.
inline bool MakeTmaF32(const void* base, int rows, int cols, CUtensorMap* out) {
  EncodeTiledFn enc = GetEncodeTiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  cuuint32_t box[2] = {(cuuint32_t)kT32BK, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// out[j, i] = in[i, j] for a row-major [rows, cols] matrix (32 x 32 tiles through shared memory).
__global__ void TransposeF32Kernel(const float* __restrict__ in, float* __restrict__ out, int rows, int cols) {
  __shared__ float t[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[i][threadIdx.x] = in[(size_t)r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[(size_t)c * rows + r] = t[threadIdx.x][i];
  }
}

// Rows from which the fp32 seam uses the tensor cores; K must give 16-byte rows for TMA.
constexpr int kTf32MinRows = 64;
inline bool Tf32Eligible(int m, int k, int n) { return m >= kTf32MinRows && n >= 16 && k % 4 == 0; }

// Splits device operands a [m,k] and bt [n,k] in place into their hi parts, writing the lo parts to a_lo /
// b_lo, then runs the three-pass tf32 GEMM into out [m,n]. All pointers are device memory, 16-byte aligned.
inline cudaError_t GemmNtTf32x3(float* a, float* a_lo, float* bt, float* b_lo, float* out, int m, int k, int n, int acc,
                                int num_sms, cudaStream_t st) {
  const size_t na = (size_t)m * k, nb = (size_t)n * k;
  SplitTf32Kernel<<<std::min<size_t>(4 * num_sms, (na + 255) / 256), 256, 0, st>>>(a, a, a_lo, na);
  SplitTf32Kernel<<<std::min<size_t>(4 * num_sms, (nb + 255) / 256), 256, 0, st>>>(bt, bt, b_lo, nb);
  CUtensorMap tah, tal, tbh, tbl;
  if (!MakeTmaF32(a, m, k, &tah) || !MakeTmaF32(a_lo, m, k, &tal) || !MakeTmaF32(bt, n, k, &tbh) ||
      !MakeTmaF32(b_lo, n, k, &tbl))
    return cudaErrorInvalidValue;
  if (!EnsureKernelAttrs((const void*)GemmNtTf32x3Kernel, kT32Smem)) return cudaErrorInvalidValue;
  const int tiles = CeilDiv(n, kT32BN) * CeilDiv(m, kT32BM);
  GemmNtTf32x3Kernel<<<std::min(tiles, num_sms), kT32Threads, kT32Smem, st>>>(tah, tal, tbh, tbl, out, m, n, k, acc);
  return cudaGetLastError();
}

}  // namespace shahd
