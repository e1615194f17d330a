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

}  // namespace shahd
