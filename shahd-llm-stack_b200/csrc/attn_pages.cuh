// Decode-row attention for long cached lengths (AttendRow, Brain/Sampling/CachedRowMath.ts:60-86, for the G
// query heads of one kv head): one CTA per (split, kv head, row). One thread of a producer warp streams the
// row's 64-position K and V blocks with bulk copies into a ring of ApStages(D) pages (blocks written by
// earlier steps are requested before griddepcontrol.wait, the block holding this step's own position after
// it); four compute warps take the pages round-robin and each keeps its own online softmax (no block-wide
// barrier per page): lane l scores positions l and l + 32 (16-byte K chunks, chunk order rotated by lane so
// the 32 lanes hit distinct banks), the page's probabilities go through a per-warp shared row, and lane l
// accumulates dims l * D/32 .. of P.V. The warps' states merge at the end (and the splits through the
// partial buffers, as the other decode attention kernels do).
#pragma once

#include "common.cuh"
#include "decode_kernels.cuh"

namespace shahd {

constexpr int kApWarps = 4;                      // compute warps
constexpr int kApThreads = (kApWarps + 1) * 32;  // + the producer warp
// automatic choice: decode steps whose rows attend at least this many cached positions on average (and whose
// rows x kv heads fill the SMs) use this kernel; shorter rows are latency-bound and go to the read-ahead kernel
constexpr int kApMinMeanLen = 384;

__host__ __device__ constexpr int ApStages(int D) { return D >= 128 ? 4 : 6; }
__host__ __device__ constexpr int ApSmemBytes(int D, int MG) {
  return ApStages(D) * 2 * kPageTokens * D * 2 +
         (MG * D + kApWarps * MG * kPageTokens + kApWarps * MG * D + 2 * kApWarps * MG + 2 * MG) * 4;
}

template <int D, int MG>
__global__ void __launch_bounds__(kApThreads) AttnPagesKernel(AttnArgs aa) {
  constexpr int NC = D / 8;    // 16-byte chunks of a K row
  constexpr int DPL = D / 32;  // output dims per lane
  constexpr int S = ApStages(D);
  constexpr int BLK = kPageTokens * D;  // elements of one K (or V) block
  extern __shared__ __align__(128) uint8_t ap_smem[];
  bf16* ring = reinterpret_cast<bf16*>(ap_smem);  // [S][K block | V block]
  float* sq = reinterpret_cast<float*>(ring + (size_t)S * 2 * BLK);  // [MG][D] pre-scaled q; later the output
  float* sp = sq + MG * D;                  // [warps][MG][64] probabilities of a warp's page
  float* wo = sp + kApWarps * MG * kPageTokens;  // [warps][MG][D]
  float* wm = wo + kApWarps * MG * D;       // [warps][MG]
  float* wl = wm + kApWarps * MG;           // [warps][MG]
  float* mm = wl + kApWarps * MG;           // [MG]
  float* ml = mm + MG;                      // [MG]
  __shared__ __align__(8) uint64_t full[S], empty[S];
  const int g = blockIdx.y, m = blockIdx.z, G = aa.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = __ldcg(aa.pos + m), slot = __ldcg(aa.slot + m);
  const int pages = p / kPageTokens + 1;
  const int pb = (int)((long long)blockIdx.x * pages / gridDim.x);
  const int np = (int)((long long)(blockIdx.x + 1) * pages / gridDim.x) - pb;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      MbarInit(&full[s], 1);
      MbarInit(&empty[s], 1);
    }
    FenceMbarInit();
  }
  __syncthreads();

  if (warp == kApWarps) {  // producer
    if (lane == 0) {
      auto issue = [&](int i) {
        const int st = i % S, pg = pb + i;
        const int len = min(kPageTokens, p + 1 - pg * kPageTokens);
        const bf16* kb = aa.kv.Block(slot, pg, aa.layer, g, 0);
        if (kb == nullptr) {  // missing page (recorded): complete the phase with no data
          MbarArrive(&full[st]);
          return;
        }
        const uint32_t bytes = (uint32_t)len * D * 2;
        MbarArriveExpectTx(&full[st], 2 * bytes);
        BulkCopyG2S(ring + (size_t)st * 2 * BLK, kb, bytes, &full[st]);
        BulkCopyG2S(ring + (size_t)st * 2 * BLK + BLK, kb + BLK, bytes, &full[st]);
      };
      int i = 0;
      // blocks wholly before the block of position p were written by earlier steps
      for (; i < np && i < S && pb + i < p / kPageTokens; i++) issue(i);
      GridDepWait();
      FenceProxyAsyncGlobal();  // the preceding kernel's K/V row at p, written by ordinary stores
      for (; i < np; i++) {
        if (i >= S && !MbarWaitBounded(&empty[i % S], (uint32_t)((i / S - 1) & 1), kWaitLimit)) {
          atomicCAS(&g_shahd_device_error, 0, kDevErrAttnTimeout);
          break;
        }
        issue(i);
      }
      // the last copies of every stage have landed before the CTA may exit
      for (int j = max(0, i - S); j < i; j++) MbarWaitBounded(&full[j % S], (uint32_t)((j / S) & 1), kWaitLimit);
    }
    GridDepLaunch();
  } else {
    GridDepWait();
    GridDepLaunch();
    const int hd = aa.H * D;
    for (int e = threadIdx.x; e < G * D; e += kApWarps * 32)
      sq[e] = __ldcg(aa.q + (size_t)m * hd + g * G * D + e) * aa.scale;
    asm volatile("bar.sync 1, %0;" ::"n"(kApWarps * 32) : "memory");  // the compute warps only
    float o[MG][DPL], mr[MG], lr[MG];
#pragma unroll
    for (int h = 0; h < MG; h++) {
      mr[h] = -INFINITY;
      lr[h] = 0.f;
#pragma unroll
      for (int j = 0; j < DPL; j++) o[h][j] = 0.f;
    }
    float* spw = sp + warp * MG * kPageTokens;
    for (int i = warp; i < np; i += kApWarps) {
      const int st = i % S, pg = pb + i;
      if (!MbarWaitBounded(&full[st], (uint32_t)((i / S) & 1), kWaitLimit)) {
        atomicCAS(&g_shahd_device_error, 0, kDevErrAttnTimeout);
        break;
      }
      const bool present = aa.kv.block_table[(size_t)slot * aa.kv.max_blocks + pg] >= 0;
      const int tv = present ? min(kPageTokens, p + 1 - pg * kPageTokens) : 0;
      const bf16* kb = ring + (size_t)st * 2 * BLK;
      const bf16* vb = kb + BLK;
      if (tv > 0) {
        float s0[MG], s1[MG];
#pragma unroll
        for (int h = 0; h < MG; h++) s0[h] = s1[h] = 0.f;
#pragma unroll
        for (int c = 0; c < NC; c++) {
          const int ch = (c + lane) % NC;
          float k0[8], k1[8];
          Bf16ChunkToFloat(*reinterpret_cast<const uint4*>(kb + (size_t)lane * D + ch * 8), k0);
          Bf16ChunkToFloat(*reinterpret_cast<const uint4*>(kb + (size_t)(lane + 32) * D + ch * 8), k1);
#pragma unroll
          for (int h = 0; h < MG; h++) {
            if (h < G) {
              const float4 qa = *reinterpret_cast<const float4*>(sq + h * D + ch * 8);
              const float4 qb = *reinterpret_cast<const float4*>(sq + h * D + ch * 8 + 4);
              const float qf[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
              for (int j = 0; j < 8; j++) {
                s0[h] = fmaf(qf[j], k0[j], s0[h]);
                s1[h] = fmaf(qf[j], k1[j], s1[h]);
              }
            }
          }
        }
        __syncwarp();  // the previous page's probabilities have been read
#pragma unroll
        for (int h = 0; h < MG; h++) {
          if (h < G) {
            const float v0 = lane < tv ? s0[h] : -INFINITY, v1 = lane + 32 < tv ? s1[h] : -INFINITY;
            const float nm = fmaxf(mr[h], WarpMax(fmaxf(v0, v1)));  // finite: position pg*64 <= p
            const float alpha = mr[h] == -INFINITY ? 0.f : __expf(mr[h] - nm);
            const float p0 = v0 == -INFINITY ? 0.f : __expf(v0 - nm);
            const float p1 = v1 == -INFINITY ? 0.f : __expf(v1 - nm);
            lr[h] = lr[h] * alpha + p0 + p1;
            mr[h] = nm;
            spw[h * kPageTokens + lane] = p0;
            spw[h * kPageTokens + lane + 32] = p1;
#pragma unroll
            for (int j = 0; j < DPL; j++) o[h][j] *= alpha;
          }
        }
        __syncwarp();
        for (int t = 0; t < tv; t++) {  // rows past tv hold stale shared memory: never read
          float vf[DPL];
          if constexpr (DPL == 2) {
            const float2 v2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vb + (size_t)t * D + 2 * lane));
            vf[0] = v2.x;
            vf[1] = v2.y;
          } else {
#pragma unroll
            for (int j = 0; j < DPL; j++) vf[j] = __bfloat162float(vb[(size_t)t * D + lane * DPL + j]);
          }
#pragma unroll
          for (int h = 0; h < MG; h++) {
            if (h < G) {
              const float pt = spw[h * kPageTokens + t];
#pragma unroll
              for (int j = 0; j < DPL; j++) o[h][j] = fmaf(pt, vf[j], o[h][j]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) MbarArrive(&empty[st]);
    }
    // this warp's state
#pragma unroll
    for (int h = 0; h < MG; h++) {
      if (h < G) {
        const float l = WarpSum(lr[h]);
        if (lane == 0) {
          wm[warp * MG + h] = mr[h];
          wl[warp * MG + h] = l;
        }
#pragma unroll
        for (int j = 0; j < DPL; j++) wo[(warp * MG + h) * D + lane * DPL + j] = o[h][j];
      }
    }
  }
  __syncthreads();
  // merge the compute warps (weights exp(m_w - M); a warp without pages has m_w = -inf)
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float M = -INFINITY, L = 0.f;
    for (int w = 0; w < kApWarps; w++) M = fmaxf(M, wm[w * MG + h]);
    for (int w = 0; w < kApWarps; w++)
      if (wm[w * MG + h] != -INFINITY) L += __expf(wm[w * MG + h] - M) * wl[w * MG + h];
    mm[h] = M;
    ml[h] = L;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int h = e / D;
    float acc = 0.f;
    for (int w = 0; w < kApWarps; w++)
      if (wm[w * MG + h] != -INFINITY) acc += __expf(wm[w * MG + h] - mm[h]) * wo[(w * MG + h) * D + e % D];
    sq[e] = acc;
  }
  __syncthreads();
  AttnFinishSplit(aa, m, g, sq, mm, ml);
}

// ---- the same page stream with the products on the tensor cores (head_dim 64) ------------------------------
// For head_dim 64 the CUDA-core kernel above spends ~1.8 K instructions per warp and page (score FMAs, bf16
// conversions, a shared-memory probability read per position and head), so with G = 4 query heads per kv head
// it is bound by issue rate, not by HBM. Here the producer copies each page's K and V blocks by TMA from the
// pool's 2-D map (64 x 64 boxes, 128-byte swizzle, so ldmatrix reads are conflict-free) and each compute warp
// runs the page as mma.sync m16n8k16 tiles with the kv head's (up to 8) query heads as the N = 8 side:
//   S^T [64 positions x 8 heads] = K [64 x 64] . Q^T      (16 mma; Q as bf16 B fragments held in registers)
//   online softmax per head on the S^T fragments (lane: heads 2t, 2t+1; shuffles across the 8 row groups)
//   P^T through a padded per-warp shared row block (bf16), then
//   O^T [64 dims x 8 heads] += V^T [64 x 64] . P^T        (16 mma; V^T by ldmatrix.trans)
// about 160 instructions per page. Positions past the row's length in its last page carry finite cache data
// (the pool is zeroed at creation and only ever holds finite K/V) and get probability 0.
struct ApMmaArgs {
  CUtensorMap kvmap;  // the KV pool as rows of 64 dims (box 64 x 64 rows, 128-byte swizzle)
  AttnArgs aa;
  int L;              // layers per page: block (page, layer, kv head, K|V) starts at row ((page*L + layer)*Hk + g)*2 + kv)*64
};
constexpr int kApmStages = 6;
constexpr int kApmBlock = kPageTokens * 64 * 2;  // bytes of one K (or V) block
constexpr int kApmPStride = kPageTokens + 8;     // bf16 per probability row: rows land on distinct banks
__host__ __device__ constexpr int ApmSmemBytes(int MG) {
  return 1024 + kApmStages * 2 * kApmBlock + kApWarps * 8 * kApmPStride * 2 +
         (MG * 64 + kApWarps * MG * 64 + 2 * kApWarps * MG + 2 * MG) * 4;
}

__device__ __forceinline__ void LdMatrixX4Trans(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}
__device__ __forceinline__ void LdMatrixX4NoTrans(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}
// D[16x8] += A[16x16] (bf16, row) . B[16x8] (bf16, col), fp32 accumulators
__device__ __forceinline__ void Mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%0, %1, %2, %3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t PackBf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int MG>
__global__ void __launch_bounds__(kApThreads) AttnPagesMmaKernel(const __grid_constant__ ApMmaArgs A) {
  constexpr int D = 64;
  constexpr int S = kApmStages;
  const AttnArgs& aa = A.aa;
  extern __shared__ uint8_t apm_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(apm_raw) + 1023) & ~uintptr_t(1023));
  bf16* sP = reinterpret_cast<bf16*>(ring + (size_t)S * 2 * kApmBlock);  // [warps][8 heads][kApmPStride]
  float* sq = reinterpret_cast<float*>(sP + kApWarps * 8 * kApmPStride);  // [MG][D] merged output
  float* wo = sq + MG * D;                   // [warps][MG][D]
  float* wm = wo + kApWarps * MG * D;        // [warps][MG]
  float* wl = wm + kApWarps * MG;            // [warps][MG]
  float* mm = wl + kApWarps * MG;            // [MG]
  float* ml = mm + MG;                       // [MG]
  __shared__ __align__(8) uint64_t full[S], empty[S];
  const int g = blockIdx.y, m = blockIdx.z, G = aa.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = __ldcg(aa.pos + m), slot = __ldcg(aa.slot + m);
  const int pages = p / kPageTokens + 1;
  const int pb = (int)((long long)blockIdx.x * pages / gridDim.x);
  const int np = (int)((long long)(blockIdx.x + 1) * pages / gridDim.x) - pb;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      MbarInit(&full[s], 1);
      MbarInit(&empty[s], 1);
    }
    FenceMbarInit();
  }
  __syncthreads();

  if (warp == kApWarps) {  // producer
    if (lane == 0) {
      PrefetchTmaDesc(&A.kvmap);
      auto issue = [&](int i) {
        const int st = i % S, pg = pb + i;
        const int page = __ldcg(aa.kv.block_table + (size_t)slot * aa.kv.max_blocks + pg);
        if (page < 0) {  // missing page (recorded): complete the phase with no data
          atomicCAS(&g_shahd_device_error, 0, kDevErrNoPage);
          MbarArrive(&full[st]);
          return;
        }
        const int row = (int)((((long long)page * A.L + aa.layer) * aa.Hk + g) * 2 * kPageTokens);
        uint8_t* dst = ring + (size_t)st * 2 * kApmBlock;
        MbarArriveExpectTx(&full[st], 2 * kApmBlock);
        TmaLoad2D(dst, &A.kvmap, &full[st], 0, row);
        TmaLoad2D(dst + kApmBlock, &A.kvmap, &full[st], 0, row + kPageTokens);
      };
      int i = 0;
      // blocks wholly before the block of position p were written by earlier steps
      for (; i < np && i < S && pb + i < p / kPageTokens; i++) issue(i);
      GridDepWait();
      FenceProxyAsyncGlobal();  // the preceding kernel's K/V row at p, written by ordinary stores
      for (; i < np; i++) {
        if (i >= S && !MbarWaitBounded(&empty[i % S], (uint32_t)((i / S - 1) & 1), kWaitLimit)) {
          atomicCAS(&g_shahd_device_error, 0, kDevErrAttnTimeout);
          break;
        }
        issue(i);
      }
      // the last copies of every stage have landed before the CTA may exit
      for (int j = max(0, i - S); j < i; j++) MbarWaitBounded(&full[j % S], (uint32_t)((j / S) & 1), kWaitLimit);
    }
    GridDepLaunch();
  } else {
    GridDepWait();
    GridDepLaunch();
    const int gq = lane >> 2, t = lane & 3;  // mma fragment row group and thread-in-group
    const int mi = lane >> 3, ri = lane & 7;  // ldmatrix: this lane's matrix and row within it
    // Q^T as B fragments (k = dims, n = heads): head gq's dims 16ks + 2t, +1 and 16ks + 8 + 2t, +1, pre-scaled
    uint32_t qb[4][2];
    {
      const float* qrow = aa.q + (size_t)m * aa.H * D + (size_t)(g * G + gq) * D;
#pragma unroll
      for (int ks = 0; ks < 4; ks++) {
        if (gq < G) {
          const float2 a = __ldcg(reinterpret_cast<const float2*>(qrow + 16 * ks + 2 * t));
          const float2 b = __ldcg(reinterpret_cast<const float2*>(qrow + 16 * ks + 8 + 2 * t));
          qb[ks][0] = PackBf16x2(a.x * aa.scale, a.y * aa.scale);
          qb[ks][1] = PackBf16x2(b.x * aa.scale, b.y * aa.scale);
        } else {
          qb[ks][0] = qb[ks][1] = 0u;
        }
      }
    }
    float o[4][4], mr[2], lr[2];
#pragma unroll
    for (int dt = 0; dt < 4; dt++)
#pragma unroll
      for (int j = 0; j < 4; j++) o[dt][j] = 0.f;
    mr[0] = mr[1] = -INFINITY;
    lr[0] = lr[1] = 0.f;
    bf16* spw = sP + warp * 8 * kApmPStride;
    for (int i = warp; i < np; i += kApWarps) {
      const int st = i % S, pg = pb + i;
      if (!MbarWaitBounded(&full[st], (uint32_t)((i / S) & 1), kWaitLimit)) {
        atomicCAS(&g_shahd_device_error, 0, kDevErrAttnTimeout);
        break;
      }
      const bool present = __ldcg(aa.kv.block_table + (size_t)slot * aa.kv.max_blocks + pg) >= 0;
      const int tv = present ? min(kPageTokens, p + 1 - pg * kPageTokens) : 0;
      if (tv > 0) {
        const uint8_t* kb = ring + (size_t)st * 2 * kApmBlock;
        const uint8_t* vb = kb + kApmBlock;
        // S^T = K . Q^T
        float sc[4][4];
#pragma unroll
        for (int mt = 0; mt < 4; mt++) {
#pragma unroll
          for (int j = 0; j < 4; j++) sc[mt][j] = 0.f;
#pragma unroll
          for (int ks = 0; ks < 4; ks++) {
            uint32_t a[4];
            LdMatrixX4NoTrans(a, SmemAddr(kb + Sw128Offset(16 * mt + ri + (mi & 1) * 8, 2 * ks + (mi >> 1))));
            Mma16816(sc[mt], a, qb[ks][0], qb[ks][1]);
          }
        }
        // online softmax per head (this lane: heads 2t, 2t+1; positions 16mt + gq and 16mt + gq + 8)
        float alpha[2], pr[4][4];
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
          float mx = -INFINITY;
#pragma unroll
          for (int mt = 0; mt < 4; mt++) {
            if (16 * mt + gq < tv) mx = fmaxf(mx, sc[mt][hh]);
            if (16 * mt + gq + 8 < tv) mx = fmaxf(mx, sc[mt][2 + hh]);
          }
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float nm = fmaxf(mr[hh], mx);  // finite: position pg*64 <= p
          alpha[hh] = mr[hh] == -INFINITY ? 0.f : __expf(mr[hh] - nm);
          float sum = 0.f;
#pragma unroll
          for (int mt = 0; mt < 4; mt++) {
            pr[mt][hh] = 16 * mt + gq < tv ? __expf(sc[mt][hh] - nm) : 0.f;
            pr[mt][2 + hh] = 16 * mt + gq + 8 < tv ? __expf(sc[mt][2 + hh] - nm) : 0.f;
            sum += pr[mt][hh] + pr[mt][2 + hh];
          }
          sum += __shfl_xor_sync(0xffffffffu, sum, 4);
          sum += __shfl_xor_sync(0xffffffffu, sum, 8);
          sum += __shfl_xor_sync(0xffffffffu, sum, 16);
          lr[hh] = lr[hh] * alpha[hh] + sum;
          mr[hh] = nm;
        }
#pragma unroll
        for (int dt = 0; dt < 4; dt++) {
          o[dt][0] *= alpha[0];
          o[dt][2] *= alpha[0];
          o[dt][1] *= alpha[1];
          o[dt][3] *= alpha[1];
        }
        // P^T as B fragments (k = positions, n = heads): through the warp's padded rows [head][position]
        __syncwarp();  // the previous page's fragments have been read
#pragma unroll
        for (int mt = 0; mt < 4; mt++) {
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            spw[(2 * t + hh) * kApmPStride + 16 * mt + gq] = __float2bfloat16_rn(pr[mt][hh]);
            spw[(2 * t + hh) * kApmPStride + 16 * mt + gq + 8] = __float2bfloat16_rn(pr[mt][2 + hh]);
          }
        }
        __syncwarp();
        // O^T += V^T . P^T
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
          const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(spw + gq * kApmPStride + 16 * ks + 2 * t);
          const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(spw + gq * kApmPStride + 16 * ks + 8 + 2 * t);
#pragma unroll
          for (int dt = 0; dt < 4; dt++) {
            uint32_t a[4];
            LdMatrixX4Trans(a, SmemAddr(vb + Sw128Offset(16 * ks + ri + (mi >> 1) * 8, 2 * dt + (mi & 1))));
            Mma16816(o[dt], a, pb0, pb1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) MbarArrive(&empty[st]);
    }
    // this warp's state: heads 2t, 2t+1, dims 16dt + gq (+ 8)
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const int h = 2 * t + hh;
      if (h < G) {
        if (gq == 0) {
          wm[warp * MG + h] = mr[hh];
          wl[warp * MG + h] = lr[hh];
        }
#pragma unroll
        for (int dt = 0; dt < 4; dt++) {
          wo[(warp * MG + h) * D + 16 * dt + gq] = o[dt][hh];
          wo[(warp * MG + h) * D + 16 * dt + gq + 8] = o[dt][2 + hh];
        }
      }
    }
  }
  __syncthreads();
  // merge the compute warps (weights exp(m_w - M); a warp without pages has m_w = -inf)
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float M = -INFINITY, L = 0.f;
    for (int w = 0; w < kApWarps; w++) M = fmaxf(M, wm[w * MG + h]);
    for (int w = 0; w < kApWarps; w++)
      if (wm[w * MG + h] != -INFINITY) L += __expf(wm[w * MG + h] - M) * wl[w * MG + h];
    mm[h] = M;
    ml[h] = L;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int h = e / D;
    float acc = 0.f;
    for (int w = 0; w < kApWarps; w++)
      if (wm[w * MG + h] != -INFINITY) acc += __expf(wm[w * MG + h] - mm[h]) * wo[(w * MG + h) * D + e % D];
    sq[e] = acc;
  }
  __syncthreads();
  AttnFinishSplit(aa, m, g, sq, mm, ml);
}

}  // namespace shahd
