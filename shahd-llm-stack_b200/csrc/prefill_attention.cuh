// Causal attention of a batched prefill (or verify) chunk over the paged cache: the attention of
// MultiHeadAttention.ForwardHidden (Brain/Nn/MultiHeadAttention.ts:46-74: MatMulNT(Q, K) ->
// CausalSoftmax(., scale) -> MatMul(., V), summed later through Wo) for every row of a chunk, in tiles.
//
// One CTA per (64-query block, kv head, sequence of the chunk): the block's queries for the group's G
// query heads stay in shared memory, the cached K/V pages 0 .. (last query's page) stream through
// shared memory once per block, and each page is scored as a 64 x 64 tile per head with an online
// softmax (running max and sum per query row, Brain/Ops/CausalSoftmax.ts:17-33 semantics: key t counts for
// query position q iff t <= q). Every query row is a row of the chunk, so the context lands where the
// per-row decode kernel would put it. The K rows were written post-RoPE by the QKV epilogue of this step.
#pragma once

#include "common.cuh"
#include "decode_kernels.cuh"

namespace shahd {

constexpr int kPfThreads = 256;
constexpr int kPfQ = 64;      // query positions per CTA
constexpr int kPfMaxG = 4;    // query heads per kv head handled by this kernel

struct PrefillAttnArgs {
  const float* q;      // [rows, H*d] post-RoPE
  float* ctx;          // [rows, H*d], or nullptr when only the bf16 copy is read
  bf16* ctxb;          // [rows, ldcb]
  int ldcb;
  KvView kv;
  int layer;
  int H, Hk, G;
  float scale;
  const int* plan;     // prefill plan [5][plan_stride]: slot, token start, length, row offset, base position
  int plan_stride, i0; // the chunk's sequences are plan entries i0 .. i0 + gridDim.z - 1
};

__host__ __device__ constexpr int PrefillAttnSmem(int D) {
  // queries [G][D][64] + K and V pages [D][64] + one score tile [64][64] + row stats [G][2][64]
  return (kPfMaxG * D * kPfQ + 2 * D * kPageTokens + kPfQ * kPageTokens + 2 * kPfMaxG * kPfQ) * 4;
}

template <int D>
__global__ void __launch_bounds__(kPfThreads) PrefillAttnKernel(PrefillAttnArgs a) {
  extern __shared__ __align__(16) float pf_smem[];
  float* sQ = pf_smem;                            // [G][D][64], pre-scaled
  float* sK = sQ + kPfMaxG * D * kPfQ;            // [D][64] (key index fastest)
  float* sV = sK + D * kPageTokens;               // [64][D]
  float* sS = sV + kPageTokens * D;               // [64 q][64 keys]
  float* sM = sS + kPfQ * kPageTokens;            // [G][64] running max
  float* sL = sM + kPfMaxG * kPfQ;                // [G][64] running sum
  GridDepWait();
  GridDepLaunch();
  const int R = a.plan_stride, e = a.i0 + blockIdx.z;
  const int slot = a.plan[e], len = a.plan[2 * R + e], base = a.plan[4 * R + e];
  const int row0 = a.plan[3 * R + e] - a.plan[3 * R + a.i0];  // the sequence's first row in the chunk
  const int qb = blockIdx.x * kPfQ;
  if (qb >= len) return;
  const int nq = min(kPfQ, len - qb);
  const int g = blockIdx.y, G = a.G, hd = a.H * D;
  const int tid = threadIdx.x;
  // queries of the block, transposed and scaled; rows past nq are zero
  for (int i = tid; i < G * D * kPfQ; i += kPfThreads) {  // consecutive threads fill consecutive words
    const int qi = i % kPfQ, dd = (i / kPfQ) % D, h = i / (kPfQ * D);
    sQ[i] = qi < nq ? a.q[(size_t)(row0 + qb + qi) * hd + (g * G + h) * D + dd] * a.scale : 0.f;
  }
  for (int i = tid; i < G * kPfQ; i += kPfThreads) {
    sM[i] = -INFINITY;
    sL[i] = 0.f;
  }
  // thread tile: query rows 4*ty .. +3, keys (scores) or dims (outputs) 4*tx .. +3
  const int ty = tid / 16, tx = tid % 16;
  constexpr int DPT = D / 16;  // output dims per thread
  float o[kPfMaxG][4][DPT];
#pragma unroll
  for (int h = 0; h < kPfMaxG; h++)
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < DPT; j++) o[h][i][j] = 0.f;
  const int qlast = base + qb + nq - 1;      // last query position of the block
  const int pages = qlast / kPageTokens + 1;  // keys 0 .. qlast
  for (int pg = 0; pg < pages; pg++) {
    const bf16* kb = a.kv.Block(slot, pg, a.layer, g, 0);
    const bf16* vb = a.kv.Block(slot, pg, a.layer, g, 1);
    const int plen = min(kPageTokens, qlast + 1 - pg * kPageTokens);  // keys of this page the block can see
    __syncthreads();  // previous page's readers are done
    for (int i = tid; i < kPageTokens * D / 8; i += kPfThreads) {
      const int t = i / (D / 8), c = (i % (D / 8)) * 8;
      float kf[8], vf[8];
      if (t < plen && kb != nullptr) {
        Bf16x8ToFloat(*reinterpret_cast<const uint4*>(kb + t * D + c), kf);
        Bf16x8ToFloat(*reinterpret_cast<const uint4*>(vb + t * D + c), vf);
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) kf[j] = vf[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        sK[(c + j) * kPageTokens + t] = kf[j];
        sV[t * D + c + j] = vf[j];
      }
    }
    __syncthreads();
    for (int h = 0; h < G; h++) {
      // scores s[q][t] for this thread's 4 x 4 tile
      float s[4][4];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) s[i][j] = 0.f;
      const float* qh = sQ + h * D * kPfQ;
#pragma unroll 8
      for (int dd = 0; dd < D; dd++) {
        const float4 qv = *reinterpret_cast<const float4*>(qh + dd * kPfQ + 4 * ty);
        const float4 kv = *reinterpret_cast<const float4*>(sK + dd * kPageTokens + 4 * tx);
        const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) s[i][j] = fmaf(qa[i], ka[j], s[i][j]);
      }
      // causal mask and the online softmax update of the tile's 4 rows (16 lanes share a row group)
      float sc[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int qpos = base + qb + 4 * ty + i;
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int tpos = pg * kPageTokens + 4 * tx + j;
          if (tpos > qpos || 4 * tx + j >= plen) s[i][j] = -INFINITY;
          mx = fmaxf(mx, s[i][j]);
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float mold = sM[h * kPfQ + 4 * ty + i];
        const float mnew = fmaxf(mold, mx);
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float p = mnew == -INFINITY ? 0.f : __expf(s[i][j] - mnew);
          sS[(4 * ty + i) * kPageTokens + 4 * tx + j] = p;
          sum += p;
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        sc[i] = mold == -INFINITY ? 0.f : __expf(mold - mnew);
        __syncwarp();
        if (tx == 0) {
          sM[h * kPfQ + 4 * ty + i] = mnew;
          sL[h * kPfQ + 4 * ty + i] = sL[h * kPfQ + 4 * ty + i] * sc[i] + sum;
        }
      }
      __syncthreads();  // the page's probabilities are in sS
      // o[q][d] = o * sc + sum_t p[q][t] v[t][d] for this thread's 4 rows x DPT dims
#pragma unroll
      for (int hh = 0; hh < kPfMaxG; hh++) {
        if (hh != h) continue;
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < DPT; j++) o[hh][i][j] *= sc[i];
        for (int t = 0; t < plen; t++) {
          float vv[DPT];
#pragma unroll
          for (int j = 0; j < DPT; j++) vv[j] = sV[t * D + tx * DPT + j];
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float p = sS[(4 * ty + i) * kPageTokens + t];
#pragma unroll
            for (int j = 0; j < DPT; j++) o[hh][i][j] = fmaf(p, vv[j], o[hh][i][j]);
          }
        }
      }
      __syncthreads();  // sS is free for the next head
    }
  }
  // normalized context rows
#pragma unroll
  for (int h = 0; h < kPfMaxG; h++) {
    if (h >= G) continue;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int qi = 4 * ty + i;
      if (qi >= nq) continue;
      const float l = sL[h * kPfQ + qi];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const size_t row = (size_t)(row0 + qb + qi);
#pragma unroll
      for (int j = 0; j < DPT; j++) {
        const int col = (g * G + h) * D + tx * DPT + j;
        const float v = o[h][i][j] * inv;
        if (a.ctx) a.ctx[row * hd + col] = v;
        a.ctxb[row * a.ldcb + col] = __float2bfloat16_rn(v);
      }
    }
  }
}

}  // namespace shahd
