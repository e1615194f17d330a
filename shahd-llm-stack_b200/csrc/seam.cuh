// Matmul-level seam of libshahd_b200: the Go FFI exports (GoKernels/ffi/matmul.go:96-395) on the GPU,
// and the device-pointer bf16 MatMulNT on the tensor cores.
#include <cstdarg>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <tuple>

#include "../../include/shahd_b200.h"
#include "common.cuh"
#include "gemm_persist.cuh"
#include "gemm_tf32.cuh"
#include "umma_linear.cuh"

namespace shahd {

int g_umma_min_rows = 17;
bool g_use_pdl = true;
int g_decode_chains = 0;  // 0 = automatic
int g_umma_prefill_attn = 1;
int g_decode_attn_kernel = 0;  // decode-row attention: 0 automatic, 1 read-ahead rows, 2 page ring, 3 page streaming  // causal prefill attention of head_dim 64 on the tensor cores
int g_persistent_step = 0;  // 1: greedy generate runs its decode steps in the persistent cluster loop
int g_fused_attn_block = 0;
int g_persist_linear = 1;  // batched prefill projections on the persistent warp-specialized tcgen05 kernel  // decode rows: norm + QKV + RoPE + attention + O projection in one launch where it fits
bool g_scalar_seam = false;  // SetScalarKernels(1): the f32 seam keeps exact fp32 FMA chains on CUDA cores

// ---- thread-local last error --------------------------------------------------------------------
static thread_local std::string t_error;

static thread_local cudaError_t t_launch_err = cudaSuccess;
static thread_local std::string t_launch_what;

void NoteLaunchError(cudaError_t e, const char* what) {
  if (t_launch_err == cudaSuccess) {
    t_launch_err = e;
    t_launch_what = what;
  }
}

cudaError_t TakeLaunchError(std::string* what) {
  const cudaError_t e = t_launch_err;
  if (what) *what = t_launch_what;
  t_launch_err = cudaSuccess;
  t_launch_what.clear();
  return e;
}

bool EnsureKernelAttrs(const void* fn, int smem_bytes, bool nonportable_cluster) {
  // The dynamic shared memory attribute is an upper limit: per (device, kernel) it only ever grows to the
  // largest request seen, so a kernel whose shared memory depends on the model shape keeps working for every
  // session after a smaller one (setting it back down would fail the larger session's launches).
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> smem_set;
  static std::set<std::pair<int, const void*>> nonportable_set;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    NoteLaunchError(cudaErrorInvalidDevice, "cudaGetDevice before setting kernel attributes");
    return false;
  }
  const auto key = std::make_pair(dev, fn);
  std::lock_guard<std::mutex> g(mu);
  cudaError_t e = cudaSuccess;
  auto it = smem_set.find(key);
  if (it == smem_set.end() || it->second < smem_bytes) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e == cudaSuccess) smem_set[key] = smem_bytes;
  }
  if (e == cudaSuccess && nonportable_cluster && !nonportable_set.count(key)) {
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess) nonportable_set.insert(key);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    NoteLaunchError(e, "cudaFuncSetAttribute");
    return false;
  }
  return true;
}

void SetError(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_error = buf;
}
const char* GetError() { return t_error.c_str(); }
void ClearError() { t_error.clear(); }

// ---- SIMT GEMM for the f32/f64 seam: C[i,j] (+)= sum_p A(i,p) B(p,j) with generic strides ---------

constexpr int kGT = 64, kGK = 16;

template <typename T>
__global__ void __launch_bounds__(256) GemmSimtKernel(const T* __restrict__ A, long long sai, long long sap,
                                                      const T* __restrict__ B, long long sbp, long long sbj,
                                                      T* __restrict__ C, int M, int N, int K, int acc) {
  __shared__ T As[kGK][kGT + 1];
  __shared__ T Bs[kGK][kGT + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int i0 = blockIdx.y * kGT, j0 = blockIdx.x * kGT;
  T accv[4][4];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 4; b++) accv[a][b] = 0;
  for (int p0 = 0; p0 < K; p0 += kGK) {
    for (int e = threadIdx.x; e < kGK * kGT; e += 256) {
      // A tile: element (i, p) with p fastest when A is K-contiguous, else i fastest
      int pi, ii;
      if (sap == 1) { pi = e % kGK; ii = e / kGK; } else { ii = e % kGT; pi = e / kGT; }
      const int gi = i0 + ii, gp = p0 + pi;
      As[pi][ii] = (gi < M && gp < K) ? A[gi * sai + gp * sap] : T(0);
      int pj, jj;
      if (sbj == 1) { jj = e % kGT; pj = e / kGT; } else { pj = e % kGK; jj = e / kGK; }
      const int gj = j0 + jj, gq = p0 + pj;
      Bs[pj][jj] = (gj < N && gq < K) ? B[gq * sbp + gj * sbj] : T(0);
    }
    __syncthreads();
#pragma unroll
    for (int p = 0; p < kGK; p++) {
      T a[4], b[4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        a[q] = As[p][ty + 16 * q];
        b[q] = Bs[p][tx + 16 * q];
      }
#pragma unroll
      for (int x = 0; x < 4; x++)
#pragma unroll
        for (int y = 0; y < 4; y++) accv[x][y] = fma(a[x], b[y], accv[x][y]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int x = 0; x < 4; x++)
#pragma unroll
    for (int y = 0; y < 4; y++) {
      const int i = i0 + ty + 16 * x, j = j0 + tx + 16 * y;
      if (i < M && j < N) {
        T* c = C + (size_t)i * N + j;
        *c = acc ? *c + accv[x][y] : accv[x][y];
      }
    }
}

// ---- per-device workspace for the host-pointer seam ---------------------------------------------
struct Workspace {
  std::mutex mu;
  void* buf = nullptr;
  size_t cap = 0;
  cudaStream_t stream = nullptr;
};

static Workspace& WorkspaceFor(int dev) {
  static Workspace ws[64];
  return ws[dev & 63];
}

// Whether the calling thread's current device is an sm_100 GPU this build runs on.
static int DeviceOk() {
  int n = 0, dev = 0, major = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) {
    cudaGetLastError();
    return 0;
  }
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return major == 10 ? 1 : 0;
}

static bool CheckDims(const char* op, long long m, long long k, long long n) {
  const char* names[3] = {"M", "K", "N"};
  long long v[3] = {m, k, n};
  for (int i = 0; i < 3; i++)
    if (v[i] < 1 || v[i] > 2147483647LL) {
      SetError("%s: dimension %s must be an integer in [1, 2147483647], got %lld", op, names[i], v[i]);
      return false;
    }
  return true;
}

enum Layout { kNN, kNT, kTN };

static int NumSMs(int dev);

static size_t Align64(size_t n) { return (n + 63) / 64 * 64; }  // 256-byte boundaries between workspace regions

template <typename T>
static void RunSeam(const char* op, Layout lay, const T* a, const T* b, T* out, int m, int k, int n, int acc) {
  ClearError();
  if (!CheckDims(op, m, k, n)) return;
  if (!a || !b || !out) {
    SetError("%s: null buffer (a native kernel cannot take a pointer to zero-length memory)", op);
    return;
  }
  if (!DeviceOk()) {
    SetError("%s: no usable sm_100 device", op);
    return;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  Workspace& w = WorkspaceFor(dev);
  std::lock_guard<std::mutex> g(w.mu);
  const size_t na = (size_t)m * k, nb = lay == kTN ? (size_t)m * n : (size_t)k * n;
  const size_t no = lay == kTN ? (size_t)k * n : (size_t)m * n;
  // f32 NT / NN with enough rows: split-TF32 tensor-core GEMM (A, A lo, B as [n,k], B lo, C, NN: B as given)
  const bool tc = sizeof(T) == 4 && lay != kTN && !g_scalar_seam && Tf32Eligible(m, k, n);
  const size_t need = tc ? (2 * Align64(na) + 2 * Align64((size_t)n * k) + Align64(no) + (lay == kNN ? Align64(nb) : 0)) *
                               sizeof(T)
                         : (na + nb + no) * sizeof(T) + 256;
  if (w.cap < need) {
    if (w.buf) cudaFree(w.buf);
    w.buf = nullptr;
    w.cap = 0;
    if (cudaMalloc(&w.buf, need) != cudaSuccess) {
      SetError("%s: cudaMalloc of %zu bytes failed", op, need);
      return;
    }
    w.cap = need;
  }
  if (!w.stream) cudaStreamCreateWithFlags(&w.stream, cudaStreamNonBlocking);
  cudaGetLastError();
  if (tc) {
    float* da = static_cast<float*>(w.buf);
    float* da_lo = da + Align64(na);
    float* dbt = da_lo + Align64(na);
    float* db_lo = dbt + Align64((size_t)n * k);
    float* dc = db_lo + Align64((size_t)n * k);
    cudaMemcpyAsync(da, a, na * 4, cudaMemcpyHostToDevice, w.stream);
    if (lay == kNT) {
      cudaMemcpyAsync(dbt, b, nb * 4, cudaMemcpyHostToDevice, w.stream);
    } else {  // MatMulF32: b is [k, n]; the GEMM wants it K-major [n, k]
      float* dbn = dc + Align64(no);
      cudaMemcpyAsync(dbn, b, nb * 4, cudaMemcpyHostToDevice, w.stream);
      TransposeF32Kernel<<<dim3(CeilDiv(n, 32), CeilDiv(k, 32)), dim3(32, 8), 0, w.stream>>>(dbn, dbt, k, n);
    }
    if (acc) cudaMemcpyAsync(dc, out, no * 4, cudaMemcpyHostToDevice, w.stream);
    cudaError_t e = GemmNtTf32x3(da, da_lo, dbt, db_lo, dc, m, k, n, acc, NumSMs(dev), w.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dc, no * 4, cudaMemcpyDeviceToHost, w.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(w.stream);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) SetError("%s: device error: %s", op, cudaGetErrorString(e));
    return;
  }
  T* da = static_cast<T*>(w.buf);
  T* db = da + na;
  T* dc = db + nb;
  cudaMemcpyAsync(da, a, na * sizeof(T), cudaMemcpyHostToDevice, w.stream);
  cudaMemcpyAsync(db, b, nb * sizeof(T), cudaMemcpyHostToDevice, w.stream);
  if (acc) cudaMemcpyAsync(dc, out, no * sizeof(T), cudaMemcpyHostToDevice, w.stream);
  int M = m, N = n, K = k;
  long long sai, sap, sbp, sbj;
  if (lay == kNN) { sai = k; sap = 1; sbp = n; sbj = 1; }
  else if (lay == kNT) { sai = k; sap = 1; sbp = 1; sbj = k; }
  else { M = k; K = m; sai = 1; sap = k; sbp = n; sbj = 1; }  // db[K,N] = aᵀ @ dout
  dim3 grid(CeilDiv(N, kGT), CeilDiv(M, kGT));
  GemmSimtKernel<T><<<grid, 256, 0, w.stream>>>(da, sai, sap, db, sbp, sbj, dc, M, N, K, acc);
  cudaMemcpyAsync(out, dc, no * sizeof(T), cudaMemcpyDeviceToHost, w.stream);
  cudaError_t e = cudaStreamSynchronize(w.stream);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) SetError("%s: device error: %s", op, cudaGetErrorString(e));
}

// ---- tcgen05 GEMM, both operands by TMA, warp-specialized, persistent: LinearPersistKernel (gemm_persist.cuh)
// with an fp32 output epilogue ----------------------------------------------------------------------------

static int NumSMs(int dev) {
  static int cache[64] = {0};
  if (!cache[dev & 63]) cudaDeviceGetAttribute(&cache[dev & 63], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev & 63];
}

int GemmNtBf16(const void* a, const void* bt, float* out, int m, int k, int n, int acc, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(bt) | reinterpret_cast<uintptr_t>(out)) & 15) {
    SetError("ShahdMatMulNTBF16Device: pointers must be 16-byte aligned");
    return SHAHD_EINVAL;
  }
  if (k % 8 != 0) {
    SetError("ShahdMatMulNTBF16Device: K=%d must be a multiple of 8 (16-byte rows for TMA)", k);
    return SHAHD_EINVAL;
  }
  LinearArgs la{};
  la.ab = static_cast<const bf16*>(a);
  la.ldab = k;
  la.a_rows = m;
  la.M = m;
  la.K = k;
  la.Kp = k;
  la.w = static_cast<const bf16*>(bt);
  la.N = n;
  TakeLaunchError(nullptr);
  LaunchPersistLinear<kNormNone, EpiF32Out>(la, EpiF32Out{out, n, acc}, st);
  std::string what;
  const cudaError_t e = TakeLaunchError(&what);
  if (e != cudaSuccess) {
    SetError("ShahdMatMulNTBF16Device: %s failed: %s", what.c_str(), cudaGetErrorString(e));
    return SHAHD_ECUDA;
  }
  return SHAHD_OK;
}

}  // namespace shahd

using namespace shahd;

extern "C" {

void MatMulF64(const double* a, const double* b, double* out, int m, int k, int n) {
  RunSeam<double>("MatMulF64", kNN, a, b, out, m, k, n, 0);
}
void MatMulNTF64(const double* a, const double* bt, double* out, int m, int k, int n, int acc) {
  RunSeam<double>("MatMulNTF64", kNT, a, bt, out, m, k, n, acc != 0);
}
void MatMulTNF64(const double* a, const double* dout, double* db, int m, int k, int n, int acc) {
  RunSeam<double>("MatMulTNF64", kTN, a, dout, db, m, k, n, acc != 0);
}
void MatMulF32(const float* a, const float* b, float* out, int m, int k, int n) {
  RunSeam<float>("MatMulF32", kNN, a, b, out, m, k, n, 0);
}
void MatMulNTF32(const float* a, const float* bt, float* out, int m, int k, int n, int acc) {
  RunSeam<float>("MatMulNTF32", kNT, a, bt, out, m, k, n, acc != 0);
}
void MatMulTNF32(const float* a, const float* dout, float* db, int m, int k, int n, int acc) {
  RunSeam<float>("MatMulTNF32", kTN, a, dout, db, m, k, n, acc != 0);
}

void SetKernelThreads(int n) { (void)n; }

int ShahdCpuSupportsAvx2Fma(void) { return DeviceOk(); }

void SetScalarKernels(int force) {
  g_umma_min_rows = force ? 0x7fffffff : 17;
  g_scalar_seam = force != 0;
}

int ShahdGpuAvailable(void) { return DeviceOk(); }

const char* ShahdLastError(void) { return GetError(); }

void ShahdSetTensorCoreMinRows(int rows) { g_umma_min_rows = rows < 1 ? 1 : rows; }

void ShahdSetProgrammaticLaunch(int enable) { g_use_pdl = enable != 0; }

void ShahdSetDecodeChains(int chains) { g_decode_chains = chains < 0 ? 0 : chains; }

void ShahdSetPersistentStep(int enable) { g_persistent_step = enable != 0; }
void ShahdSetTensorCorePrefillAttention(int enable) { g_umma_prefill_attn = enable != 0; }
void ShahdSetDecodeAttentionKernel(int mode) { g_decode_attn_kernel = mode < 0 || mode > 3 ? 0 : mode; }
void ShahdSetFusedAttentionBlock(int enable) { g_fused_attn_block = enable != 0; }
void ShahdSetPersistentPrefillProjections(int enable) { g_persist_linear = enable != 0; }

int ShahdDeviceErrorFlag(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_shahd_device_error, sizeof(int)) != cudaSuccess) return -1;
  return v;
}

int ShahdMatMulNTF32Device(const float* a, const float* bt, float* out, int m, int k, int n, int acc, void* stream) {
  const char* op = "ShahdMatMulNTF32Device";
  ClearError();
  if (!CheckDims(op, m, k, n)) return SHAHD_EINVAL;
  if (!a || !bt || !out) {
    SetError("%s: null pointer", op);
    return SHAHD_EINVAL;
  }
  if ((reinterpret_cast<uintptr_t>(out) & 15) || k % 4 != 0) {
    SetError("%s: out must be 16-byte aligned and K a multiple of 4 (16-byte rows for TMA), got K=%d", op, k);
    return SHAHD_EINVAL;
  }
  if (!DeviceOk()) {
    SetError("%s: no usable sm_100 device", op);
    return SHAHD_ENODEV;
  }
  int dev = 0;
  SHAHD_CUDA_TRY(cudaGetDevice(&dev));
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  Workspace& w = WorkspaceFor(dev);
  std::lock_guard<std::mutex> g(w.mu);
  const size_t na = Align64((size_t)m * k), nb = Align64((size_t)n * k);
  const size_t need = 2 * (na + nb) * sizeof(float);
  if (w.cap < need) {
    SHAHD_CUDA_TRY(cudaStreamSynchronize(st));  // the old workspace may still be read by queued work
    if (w.buf) cudaFree(w.buf);
    w.buf = nullptr;
    w.cap = 0;
    SHAHD_CUDA_TRY(cudaMalloc(&w.buf, need));
    w.cap = need;
  }
  float* ah = static_cast<float*>(w.buf);
  float* al = ah + na;
  float* bh = al + na;
  float* bl = bh + nb;
  // the caller's operands stay untouched: the split reads them and writes both parts to the workspace
  const size_t ea = (size_t)m * k, eb = (size_t)n * k;
  SplitTf32Kernel<<<std::min<size_t>(4 * NumSMs(dev), (ea + 255) / 256), 256, 0, st>>>(a, ah, al, ea);
  SplitTf32Kernel<<<std::min<size_t>(4 * NumSMs(dev), (eb + 255) / 256), 256, 0, st>>>(bt, bh, bl, eb);
  CUtensorMap tah, tal, tbh, tbl;
  if (!MakeTmaF32(ah, m, k, &tah) || !MakeTmaF32(al, m, k, &tal) || !MakeTmaF32(bh, n, k, &tbh) ||
      !MakeTmaF32(bl, n, k, &tbl)) {
    SetError("%s: cuTensorMapEncodeTiled failed", op);
    return SHAHD_ECUDA;
  }
  if (!EnsureKernelAttrs((const void*)GemmNtTf32x3Kernel, kT32Smem)) {
    TakeLaunchError(nullptr);
    SetError("%s: the GEMM kernel's shared-memory limit could not be set", op);
    return SHAHD_ECUDA;
  }
  const int tiles = CeilDiv(n, kT32BN) * CeilDiv(m, kT32BM);
  GemmNtTf32x3Kernel<<<std::min(tiles, NumSMs(dev)), kT32Threads, kT32Smem, st>>>(tah, tal, tbh, tbl, out, m, n, k, acc);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    SetError("%s: launch failed: %s", op, cudaGetErrorString(e));
    return SHAHD_ECUDA;
  }
  return SHAHD_OK;
}

int ShahdMatMulNTBF16Device(const void* a, const void* bt, float* out, int m, int k, int n, int acc, void* stream) {
  ClearError();
  if (!CheckDims("ShahdMatMulNTBF16Device", m, k, n)) return SHAHD_EINVAL;
  if (!a || !bt || !out) {
    SetError("ShahdMatMulNTBF16Device: null pointer");
    return SHAHD_EINVAL;
  }
  return GemmNtBf16(a, bt, out, m, k, n, acc, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
