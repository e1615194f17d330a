// Shared helpers for the sm_100a kernels of libshahd_b200: error plumbing, bf16 conversion, warp
// reductions, and the inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor) and tcgen05.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

namespace shahd {

// ---- host-side error recording (thread-local last error, like a status + message pair) ----------
void SetError(const char* fmt, ...);
const char* GetError();
void ClearError();

#define SHAHD_CUDA_TRY(expr)                                                                      \
  do {                                                                                            \
    cudaError_t err_ = (expr);                                                                    \
    if (err_ != cudaSuccess) {                                                                    \
      ::shahd::SetError("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(err_), __FILE__, __LINE__); \
      return SHAHD_ECUDA;                                                                         \
    }                                                                                             \
  } while (0)

using bf16 = __nv_bfloat16;

// Kernel launches of a decode step use programmatic dependent launch: the next kernel is scheduled while
// its predecessor drains and runs its independent prologue (barrier init, TMEM allocation, weight loads)
// before GridDepWait(). Process-wide switch, on by default.
extern bool g_use_pdl;

// First launch failure on this thread since the last TakeLaunchError() (a kernel that did not launch, or
// could not be prepared, e.g. a tensor map that failed to encode). Launch helpers record into it instead of
// returning silently, and every entry point that enqueues kernels checks it before reporting success.
void NoteLaunchError(cudaError_t e, const char* what);
cudaError_t TakeLaunchError(std::string* what);

// Sets a kernel's dynamic shared memory limit (and, optionally, non-portable cluster sizes) once per
// (device, kernel): function attributes belong to the device's context, and sessions on several devices
// may run in one process. Thread-safe. Returns false (and records the failure) when the runtime refuses.
bool EnsureKernelAttrs(const void* fn, int smem_bytes, bool nonportable_cluster = false);

template <typename... KArgs, typename... Args>
inline void LaunchPdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_use_pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) NoteLaunchError(e, "kernel launch");
}

// LaunchPdl with the CTAs grouped into thread-block clusters of `cluster` (grid divisible by it).
template <typename... KArgs, typename... Args>
inline void LaunchPdlCluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, dim3 cluster, cudaStream_t st,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster.x;
  attr[0].val.clusterDim.y = cluster.y;
  attr[0].val.clusterDim.z = cluster.z;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_use_pdl ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) NoteLaunchError(e, "cluster kernel launch");
}

__host__ __device__ inline int CeilDiv(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline int RoundUp(int a, int b) { return CeilDiv(a, b) * b; }

// ---- device helpers ------------------------------------------------------------------------------

__device__ __forceinline__ float WarpSum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float WarpMax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Eight bf16 packed in a uint4 -> eight floats.
__device__ __forceinline__ void Bf16x8ToFloat(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 LoadNc16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Argmax candidate merge with ArgmaxOf's rule (Brain/Sampling/Distribution.ts:19-30): the larger value
// wins, equal values keep the smaller index; NaN never wins. idx == INT_MAX means "no candidate".
__device__ __forceinline__ void ArgmaxMerge(float& bv, int& bi, float v, int i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

// ---- programmatic dependent launch ---------------------------------------------------------------
// Wait until every prerequisite grid has completed and its memory is visible (a no-op when the kernel
// was launched without the programmatic-serialization attribute).
__device__ __forceinline__ void GridDepWait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the dependent grid to be scheduled; it still waits for this grid's completion in GridDepWait.
__device__ __forceinline__ void GridDepLaunch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Orders this thread's later async-proxy reads (TMA, bulk copies) after generic-proxy writes it may now
// observe, such as a predecessor grid's stores seen through GridDepWait.
__device__ __forceinline__ void FenceProxyAsyncGlobal() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Thread-block clusters: a barrier over every thread of the cluster (release/acquire: shared-memory
// writes before it are visible to all CTAs of the cluster after it), and a 16-byte load from the shared
// memory of CTA `rank` at the address of `p` in this CTA's window.
__device__ __forceinline__ void ClusterSync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float4 LoadPeerF32x4(const float* p, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  uint32_t ra;
  float4 v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(ra)
               : "memory");
  return v;
}

// ---- shared-memory address, mbarrier, TMA, tcgen05 (inline PTX, sm_100a) -------------------------

__device__ __forceinline__ uint32_t SmemAddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void MbarInit(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(SmemAddr(bar)), "r"(count));
}

__device__ __forceinline__ void FenceMbarInit() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void MbarArriveExpectTx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(SmemAddr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void MbarArrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(SmemAddr(bar)) : "memory");
}

// One probe of the barrier's phase `parity`; true once that phase has completed.
__device__ __forceinline__ bool MbarTryWait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(SmemAddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` probes (each probe itself suspends for a hardware-chosen time)
// and returns false, so a lost arrival turns into an error status instead of a hung GPU.
__device__ __forceinline__ bool MbarWaitBounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; i++)
    if (MbarTryWait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void FenceProxyAsyncShared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2-D tiled TMA load global -> shared, completion counted on `bar` (no multicast).
__device__ __forceinline__ void TmaLoad2D(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          SmemAddr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(SmemAddr(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void PrefetchTmaDesc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// TMEM allocation (one full warp executes these).
__device__ __forceinline__ void TmemAlloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(SmemAddr(smem_slot)), "r"(ncols));
}
__device__ __forceinline__ void TmemRelinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;"); }
__device__ __forceinline__ void TmemDealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void TcgenFenceBefore() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void TcgenFenceAfter() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] · B[smem]ᵀ, kind::f16 (bf16 inputs, fp32 accumulate), issued by one thread.
__device__ __forceinline__ void UmmaBf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void UmmaCommit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(SmemAddr(bar)) : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread: thread t of warp w reads TMEM lane 32*(w%4)+t.
__device__ __forceinline__ void TmemLoad16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// The same with 8 consecutive columns per thread.
__device__ __forceinline__ void TmemLoad8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void TmemWaitLd() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand in the 128-byte-swizzle canonical layout:
// rows of 64 bf16 (128 B), 8-row atoms of 1024 B stacked at SBO = 1024 B; LBO unused (1); version 1
// (bits 46-47); layout type 2 = SWIZZLE_128B (bits 61-63). The start address must sit in a
// 1024-byte-aligned atom (plus the 32-byte K advance inside the atom).
__device__ __forceinline__ uint64_t SmemDescSw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;             // LBO (ignored for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // SBO
  d |= (uint64_t)1 << 46;             // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: bf16 A/B, fp32 D, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t UmmaIdescBf16(int M, int N) {
  return (1u << 4)                        // D format F32
         | (1u << 7)                      // A format BF16
         | (1u << 10)                     // B format BF16
         | ((uint32_t)(N >> 3) << 17)     // N >> 3
         | ((uint32_t)(M >> 4) << 24);    // M >> 4
}

// Byte offset of the 16-byte chunk `c` (0..7) of row `r` inside a SWIZZLE_128B K-major tile whose rows
// are 128 B: chunks are XOR-permuted by the row's position inside its 8-row atom.
__host__ __device__ inline uint32_t Sw128Offset(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

}  // namespace shahd
