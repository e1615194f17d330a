// The single translation unit of libshahd_b200.so: one device module, so the kernels share one
// g_shahd_device_error flag and one set of template instantiations.
#include "seam.cuh"
#include "session.cuh"
#include "attention_op.cuh"

// ---- MatMulNTF32 without device allocation ------------------------------------------------------
// MatMulNTF32 stages its operands in a per-device workspace that it grows with cudaFree + cudaMalloc
// whenever a call needs more room. Two kinds of caller cannot accept that: a process whose device
// memory is already committed (a decode session whose KV page pool was sized to fill HBM, so any
// cudaMalloc fails), and a caller that must not stall other streams (cudaFree waits for the whole
// device, so growing the workspace would hold up decode steps running on other threads).
// ShahdMatMulNTF32NoAlloc runs the same GEMM kernel on operands staged in the fixed array below,
// which is part of the library's device image, so a call never allocates or frees device memory.

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr size_t kNoAllocAlignFloats = 64;                 // each operand starts on a 256-byte boundary

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

static std::mutex g_noalloc_setup_mu;
static float* g_noalloc_ptr[64];  // device address of g_noalloc_scratch, looked up once per device

// Looks the array's device address up for the current device (the first call on each device does this;
// it also makes the runtime load the library's device module on that device if nothing has yet). The
// address belongs to the device's primary context, the one the CUDA runtime uses: callers that make some
// other context current on the device are not supported.
static float* NoAllocScratch(int dev) {
  std::lock_guard<std::mutex> g(g_noalloc_setup_mu);
  if (g_noalloc_ptr[dev & 63]) return g_noalloc_ptr[dev & 63];
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    SetError("ShahdMatMulNTF32NoAlloc: cudaGetSymbolAddress of the scratch array failed on device %d: %s", dev,
             cudaGetErrorString(e));
    return nullptr;
  }
  g_noalloc_ptr[dev & 63] = static_cast<float*>(p);
  return g_noalloc_ptr[dev & 63];
}

static size_t RoundUpFloats(size_t n) { return (n + kNoAllocAlignFloats - 1) / kNoAllocAlignFloats * kNoAllocAlignFloats; }

extern "C" int ShahdMatMulNTF32NoAlloc(const float* a, const float* bt, float* out, int m, int k, int n, int acc) {
  const char* op = "ShahdMatMulNTF32NoAlloc";
  ClearError();
  cudaGetLastError();  // a stale error of an earlier runtime call on this thread is not this call's failure
  if (!CheckDims(op, m, k, n)) return SHAHD_EINVAL;
  if (!a || !bt || !out) {
    SetError("%s: null buffer", op);
    return SHAHD_EINVAL;
  }
  const size_t na = RoundUpFloats((size_t)m * k), nb = RoundUpFloats((size_t)n * k), no = (size_t)m * n;
  const size_t need = (na + nb + no) * sizeof(float);
  if (need > kNoAllocScratchBytes) {
    SetError("%s: operands need %zu bytes of scratch (A %dx%d, B %dx%d, C %dx%d f32); the fixed limit is %zu bytes",
             op, need, m, k, n, k, m, n, kNoAllocScratchBytes);
    return SHAHD_EINVAL;
  }
  if (!DeviceOk()) {
    SetError("%s: no usable sm_100 device", op);
    return SHAHD_ENODEV;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    SetError("%s: cudaGetDevice failed", op);
    return SHAHD_ECUDA;
  }
  float* base = NoAllocScratch(dev);
  if (!base) return SHAHD_ECUDA;
  float* da = base;
  float* db = da + na;
  float* dc = db + nb;
  // The per-thread default stream: no stream is created, and calls from different threads do not
  // serialize behind one another. Nothing in the scratch has to start at zero: A and B are uploaded on
  // every call, C is uploaded when acc != 0 and otherwise fully written by the kernel.
  const cudaStream_t st = cudaStreamPerThread;
  const char* step = "copying A to the device";
  cudaError_t e = cudaMemcpyAsync(da, a, (size_t)m * k * sizeof(float), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    step = "copying B to the device";
    e = cudaMemcpyAsync(db, bt, (size_t)n * k * sizeof(float), cudaMemcpyHostToDevice, st);
  }
  if (e == cudaSuccess && acc) {
    step = "copying C to the device";
    e = cudaMemcpyAsync(dc, out, no * sizeof(float), cudaMemcpyHostToDevice, st);
  }
  if (e == cudaSuccess) {
    step = "launching the GEMM";
    dim3 grid(CeilDiv(n, kGT), CeilDiv(m, kGT));
    GemmSimtKernel<float><<<grid, 256, 0, st>>>(da, k, 1, db, 1, k, dc, m, n, k, acc);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    step = "copying C back";
    e = cudaMemcpyAsync(out, dc, no * sizeof(float), cudaMemcpyDeviceToHost, st);
  }
  if (e == cudaSuccess) {
    step = "waiting for the device";
    e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) {
    SetError("%s: %s failed: %s", op, step, cudaGetErrorString(e));
    return SHAHD_ECUDA;
  }
  return SHAHD_OK;
}
