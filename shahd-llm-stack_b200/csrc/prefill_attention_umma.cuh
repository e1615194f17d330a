// Causal prefill attention on the tensor cores (head_dim 64): the attention of
// MultiHeadAttention.ForwardHidden (Brain/Nn/MultiHeadAttention.ts:46-74: MatMulNT(Q, K) ->
// CausalSoftmax(., scale) (Brain/Ops/CausalSoftmax.ts:17-33) -> MatMul(., V)) for every row of a prefill
// chunk, over the paged cache.
//
// One CTA per (128-query block, query head, sequence of the chunk); 6 warps:
//   warps 0-3  one query row per thread (TMEM lane = row): the block's queries into shared memory as the
//              bf16 A operand, then per 64-position page the online softmax of the row's scores, the bf16
//              probabilities as the A operand of P.V (two alternating buffers, so page j's probabilities
//              are written while page j-1's P.V still reads its own), and the fp32 context accumulated in
//              registers;
//   warp 4     one thread issues the MMAs: S = Q.K^T (M 128, N 64 keys, K 64 dims) into TMEM columns 0-63
//              or 64-127 (alternating: page j+1's scores are computed while the softmax warps work on
//              page j), O_page = P.V (M 128, N 64 dims, K 64 keys) into columns 128-191 or 192-255
//              (alternating, so the softmax warps read one page's O while the next page's is computed);
//   warp 5     one thread streams the kv head's K and V blocks of every page the block can see by TMA
//              (128-byte swizzle, a 3-stage ring; this GPU's own memory, no multicast).
// K blocks are the K-major B operand of S; V blocks ([position][dim], dims contiguous) are the MN-major B
// operand of P.V. Key t counts for query position q iff t <= q (CausalSoftmax). Running max and sum per row
// in fp32 (exp of (s - max) * scale); the context is normalized once at the end.
#pragma once

#include "common.cuh"
#include "decode_kernels.cuh"
#include "prefill_attention.cuh"

namespace shahd {

constexpr int kFaQ = 128;                        // query rows per CTA (one query head)
constexpr int kFaD = 64;                         // head_dim served
constexpr int kFaStages = 3;                     // K/V ring depth (pages)
constexpr int kFaThreads = 192;                  // 4 softmax warps, 1 MMA warp, 1 TMA warp
constexpr uint32_t kFaTmemCols = 256;            // two S pages + two O pages, 64 columns each
constexpr int kFaBlock = kPageTokens * kFaD * 2;  // one K or V block of a page: 64 positions x 64 dims, bf16
constexpr int kFaTile = kFaQ * kFaD * 2;         // the Q or P operand: 128 rows x 128 B

struct FaShared {
  uint64_t kv_full[kFaStages], kv_empty[kFaStages];
  uint64_t q_ready, s_full[2], p_ready, o_full[2];  // s_full[b] / o_full[b]: pages j with j & 1 == b
  uint32_t tmem;
  volatile int abort;
};

// Q | P[2] | ring of (K, V) blocks | barriers; 1024-byte aligned base for the swizzled tiles. Sized so that
// at most two CTAs share an SM (their TMEM allocations then always fit the SM's 512 columns).
constexpr int kFaSmemBytes = 1024 + 3 * kFaTile + kFaStages * 2 * kFaBlock + 256;
constexpr int kFaSmemLaunch = kFaSmemBytes > 100 * 1024 ? kFaSmemBytes : 100 * 1024;

struct FaArgs {
  CUtensorMap kvmap;  // the KV pool as rows of 64 dims (box 64 x 64 rows, 128-byte swizzle)
  PrefillAttnArgs a;  // rows, context outputs, cache, plan (the SIMT kernel's arguments)
  int L;              // layers: page block (page, layer, kv head, K|V) starts at row ((page*L + layer)*Hk + g)*2 + kv) * 64
  int qblocks;        // 128-query blocks of the chunk's longest sequence
};

// Matrix descriptor of an MN-major operand in the 128-byte-swizzle layout: rows of 128 B hold 64 consecutive
// MN elements, 8-row groups along K are 1024 B apart (stride byte offset); a single 64-element group along
// MN, so the leading byte offset is unused.
__device__ __forceinline__ uint64_t SmemDescSw128Mn(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)(8192 >> 4) << 16;  // LBO: next 64-element group along MN (none here)
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO: next 8 rows along K
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 bits, 32 consecutive columns per thread.
__device__ __forceinline__ void TmemLoad32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Records a bounded wait that gave up; every role then leaves its loop.
__device__ __forceinline__ bool FaWait(FaShared* sh, uint64_t* bar, uint32_t parity) {
  if (MbarWaitBounded(bar, parity, kWaitLimit)) return true;
  atomicCAS(&g_shahd_device_error, 0, kDevErrAttnTimeout);
  sh->abort = 1;
  return false;
}

__global__ void __launch_bounds__(kFaThreads) PrefillAttnUmmaKernel(const __grid_constant__ FaArgs A) {
  extern __shared__ uint8_t fa_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sP = base + kFaTile;        // P of page j at sP + (j & 1) * kFaTile
  uint8_t* ring = base + 3 * kFaTile;  // stage s: K block at ring + 2s*kFaBlock, V block right after
  FaShared* sh = reinterpret_cast<FaShared*>(ring + kFaStages * 2 * kFaBlock);
  const PrefillAttnArgs& a = A.a;
  GridDepWait();
  const int R = a.plan_stride, e = a.i0 + blockIdx.z;
  const int slot = a.plan[e], len = a.plan[2 * R + e], basepos = a.plan[4 * R + e];
  const int row0 = a.plan[3 * R + e] - a.plan[3 * R + a.i0];  // the sequence's first row in the chunk
  const int qb = (A.qblocks - 1 - (int)blockIdx.x) * kFaQ;    // the longest (latest) blocks start first
  if (qb >= len) return;
  const int nq = min(kFaQ, len - qb);
  const int h = blockIdx.y, g = h / a.G;
  const int npages = (basepos + qb + nq - 1) / kPageTokens + 1;  // keys 0 .. the block's last query
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFaStages; s++) {
      MbarInit(&sh->kv_full[s], 1);
      MbarInit(&sh->kv_empty[s], 1);
    }
    MbarInit(&sh->q_ready, kFaQ);
    MbarInit(&sh->s_full[0], 1);
    MbarInit(&sh->s_full[1], 1);
    MbarInit(&sh->p_ready, kFaQ);
    MbarInit(&sh->o_full[0], 1);
    MbarInit(&sh->o_full[1], 1);
    sh->abort = 0;
    FenceMbarInit();
  }
  if (warp == 0) {
    TmemAlloc(&sh->tmem, kFaTmemCols);
    TmemRelinquish();
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  const uint32_t tmem = sh->tmem;
  // dependents may be scheduled only once this CTA holds its TMEM: a dependent CTA that took the SM's
  // columns first would wait for this grid while this CTA waited for its columns
  GridDepLaunch();

  if (warp == 5) {
    if (lane == 0) {  // TMA producer: K and V blocks of pages 0 .. npages-1
      PrefetchTmaDesc(&A.kvmap);
      int issued = 0;
      for (int j = 0; j < npages && !sh->abort; j++) {
        const int st = j % kFaStages;
        if (j >= kFaStages && !FaWait(sh, &sh->kv_empty[st], (uint32_t)((j / kFaStages - 1) & 1))) break;
        int page = a.kv.block_table[(size_t)slot * a.kv.max_blocks + j];
        if (page < 0) {  // the host assigns every page before the launch; keep the copy in bounds regardless
          atomicCAS(&g_shahd_device_error, 0, kDevErrNoPage);
          page = 0;
        }
        const int row = (int)((((long long)page * A.L + a.layer) * a.Hk + g) * 2 * kPageTokens);
        uint8_t* dst = ring + (size_t)st * 2 * kFaBlock;
        MbarArriveExpectTx(&sh->kv_full[st], 2 * kFaBlock);
        TmaLoad2D(dst, &A.kvmap, &sh->kv_full[st], 0, row);
        TmaLoad2D(dst + kFaBlock, &A.kvmap, &sh->kv_full[st], 0, row + kPageTokens);
        issued = j + 1;
      }
      // every issued copy lands before the CTA may exit (the last phase of each stage's barrier)
      for (int j = max(0, issued - kFaStages); j < issued; j++)
        MbarWaitBounded(&sh->kv_full[j % kFaStages], (uint32_t)((j / kFaStages) & 1), kWaitLimit);
    }
  } else if (warp == 4) {
    if (lane == 0) {  // MMA issue
      const uint32_t idesc_s = UmmaIdescBf16(kFaQ, kPageTokens);
      const uint32_t idesc_pv = UmmaIdescBf16(kFaQ, kFaD) | (1u << 16);  // B (V) MN-major
      const uint64_t qdesc = SmemDescSw128(SmemAddr(sQ));
      const uint64_t pdesc0 = SmemDescSw128(SmemAddr(sP));
      // S of page j into TMEM columns 64 * (j & 1), committed to s_full[j & 1]
      auto issue_s = [&](int j) -> bool {
        const int st = j % kFaStages;
        if (!FaWait(sh, &sh->kv_full[st], (uint32_t)((j / kFaStages) & 1))) return false;
        TcgenFenceAfter();
        const uint64_t kdesc = SmemDescSw128(SmemAddr(ring + (size_t)st * 2 * kFaBlock));
        for (int kk = 0; kk < kFaD / 16; kk++)
          UmmaBf16(tmem + 64u * (uint32_t)(j & 1), qdesc + (uint64_t)(2 * kk), kdesc + (uint64_t)(2 * kk), idesc_s,
                   kk > 0 ? 1u : 0u);
        UmmaCommit(&sh->s_full[j & 1]);
        return true;
      };
      bool ok = FaWait(sh, &sh->q_ready, 0);
      TcgenFenceAfter();
      ok = ok && issue_s(0) && (npages < 2 || issue_s(1));
      for (int j = 0; j < npages && ok; j++) {
        const int st = j % kFaStages;
        if (!FaWait(sh, &sh->p_ready, (uint32_t)(j & 1))) break;
        TcgenFenceAfter();
        const uint64_t vdesc = SmemDescSw128Mn(SmemAddr(ring + (size_t)st * 2 * kFaBlock + kFaBlock));
        const uint32_t ocol = tmem + 128u + 64u * (uint32_t)(j & 1);
        const uint64_t pdesc = pdesc0 + (uint64_t)((j & 1) * (kFaTile >> 4));
        for (int kk = 0; kk < kPageTokens / 16; kk++)  // 16 keys = two 8-row groups of V per step
          UmmaBf16(ocol, pdesc + (uint64_t)(2 * kk), vdesc + (uint64_t)(kk * (2048 >> 4)), idesc_pv,
                   kk > 0 ? 1u : 0u);
        UmmaCommit(&sh->o_full[j & 1]);
        UmmaCommit(&sh->kv_empty[st]);
        // the softmax warps have read page j's scores (p_ready): its S columns take page j + 2
        if (j + 2 < npages) ok = issue_s(j + 2);
      }
    }
  } else {  // softmax warps: thread = query row = TMEM lane
    const int qi = threadIdx.x;
    const int hd = a.H * kFaD;
    const size_t row = (size_t)(row0 + qb + qi);
    {  // the query row as bf16 (rows past nq are zero)
      const float* qrow = a.q + row * hd + h * kFaD;
#pragma unroll
      for (int c = 0; c < 8; c++) {
        float v[8];
        if (qi < nq) {
          const float4 v0 = *reinterpret_cast<const float4*>(qrow + 8 * c);
          const float4 v1 = *reinterpret_cast<const float4*>(qrow + 8 * c + 4);
          v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w; v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
        } else {
#pragma unroll
          for (int t = 0; t < 8; t++) v[t] = 0.f;
        }
        StoreNbf<8>(reinterpret_cast<bf16*>(sQ + Sw128Offset(qi, c)), v);
      }
      FenceProxyAsyncShared();
      MbarArrive(&sh->q_ready);
    }
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const int qpos = basepos + qb + qi;
    const float scale = a.scale;
    float o[kFaD];
#pragma unroll
    for (int c = 0; c < kFaD; c++) o[c] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    for (int j = 0; j < npages && ok; j++) {
      ok = FaWait(sh, &sh->s_full[j & 1], (uint32_t)((j >> 1) & 1));
      if (!ok) break;
      TcgenFenceAfter();
      uint32_t u[kPageTokens];
      const uint32_t scol = lane_base + 64u * (uint32_t)(j & 1);
      TmemLoad32(scol, u);
      TmemLoad32(scol + 32u, u + 32);
      TmemWaitLd();
      float p[kPageTokens];
      float mx = m;
      const int t0 = j * kPageTokens;
#pragma unroll
      for (int c = 0; c < kPageTokens; c++) {
        p[c] = (t0 + c <= qpos) ? __uint_as_float(u[c]) : -INFINITY;
        mx = fmaxf(mx, p[c]);
      }
      const float alpha = (m == -INFINITY) ? 0.f : __expf((m - mx) * scale);
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < kPageTokens; c++) {
        p[c] = (mx == -INFINITY || p[c] == -INFINITY) ? 0.f : __expf((p[c] - mx) * scale);
        rs += p[c];
      }
      l = l * alpha + rs;
      m = mx;
      // P buffer j & 1 was last read by page j-2's P.V, whose completion this thread saw at page j-1
#pragma unroll
      for (int c = 0; c < 8; c++)
        StoreNbf<8>(reinterpret_cast<bf16*>(sP + (j & 1) * kFaTile + Sw128Offset(qi, c)), p + 8 * c);
      FenceProxyAsyncShared();
      // page j-1's P.V complete: every thread has arrived for page j-1, so this thread's arrival below
      // counts toward page j's phase of p_ready (a thread running a page ahead would complete the wrong
      // phase), and its O page may be read
      if (j > 0) {
        ok = FaWait(sh, &sh->o_full[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1));
        if (!ok) break;
      }
      TcgenFenceBefore();
      MbarArrive(&sh->p_ready);
      if (j > 0) {  // o = o * alpha(j-1) + O_page(j-1) (the current page's P.V writes the other O buffer)
        TcgenFenceAfter();
        const uint32_t ocol = lane_base + 128u + 64u * (uint32_t)((j - 1) & 1);
        TmemLoad32(ocol, u);
        TmemLoad32(ocol + 32u, u + 32);
        TmemWaitLd();
#pragma unroll
        for (int c = 0; c < kFaD; c++) o[c] = o[c] * alpha_prev + __uint_as_float(u[c]);
      }
      alpha_prev = alpha;
    }
    if (ok && FaWait(sh, &sh->o_full[(npages - 1) & 1], (uint32_t)(((npages - 1) >> 1) & 1))) {
      TcgenFenceAfter();
      uint32_t u[kFaD];
      const uint32_t ocol = lane_base + 128u + 64u * (uint32_t)((npages - 1) & 1);
      TmemLoad32(ocol, u);
      TmemLoad32(ocol + 32u, u + 32);
      TmemWaitLd();
#pragma unroll
      for (int c = 0; c < kFaD; c++) o[c] = o[c] * alpha_prev + __uint_as_float(u[c]);
      if (qi < nq) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int c = 0; c < kFaD; c++) o[c] *= inv;
        const int col = h * kFaD;
        if (a.ctx) {
          float4* dst = reinterpret_cast<float4*>(a.ctx + row * hd + col);
#pragma unroll
          for (int c = 0; c < kFaD / 4; c++) dst[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
        }
        StoreNbf<kFaD>(a.ctxb + row * a.ldcb + col, o);
      }
    }
  }
  TcgenFenceBefore();
  __syncthreads();
  TcgenFenceAfter();
  if (warp == 0) TmemDealloc(tmem, kFaTmemCols);
}

}  // namespace shahd
