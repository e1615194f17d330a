// Decode-step kernels for one batched cached step over M rows (row r = one sequence's next token).
// Restates AdvanceOneToken + HeadLogitsRow (Brain/Sampling/CachedForward.ts:32-96,
// CachedRowMath.ts:14-137) as: embed -> per layer [norm+QKV+RoPE+KV append] -> [attention over the
// paged cache] -> [O projection + residual] -> [norm + gate/up + SwiGLU/GeGLU | fc + ReLU] ->
// [down projection + residual] -> [final norm + LM head + argmax partials] -> finish.
#pragma once

#include "common.cuh"

namespace shahd {

__device__ int g_shahd_device_error;  // 0 = ok; otherwise the first kDevErr* code recorded
constexpr int kDevErrUmmaTimeout = 1;
constexpr int kDevErrGemmTimeout = 2;
constexpr int kDevErrNoPage = 3;

constexpr int kPageTokens = 64;  // positions per KV page (and per attention chunk)

enum NormKind { kNormNone = 0, kNormRms = 1, kNormLayer = 2 };

// Paged KV pool: page = [layer][kv head][K|V][64 positions][head_dim] bf16, K stored after RoPE
// (KvCache.ts:1-15). block_table[slot * max_blocks + pos / 64] names the page holding `pos`.
struct KvView {
  bf16* pool;
  const int* block_table;
  int max_blocks;
  int Hk;
  int d;
  size_t page_elems;
  // Element offset of (slot, pos, layer, kv head, K|V), or -1 when no page backs `pos` (the host assigns
  // pages before every launch; a miss is recorded as kDevErrNoPage and the access is skipped).
  __device__ __forceinline__ long long Offset(int slot, int pos, int layer, int g, int kv) const {
    const int page = block_table[slot * max_blocks + (pos >> 6)];
    if (page < 0) {
      atomicCAS(&g_shahd_device_error, 0, kDevErrNoPage);
      return -1;
    }
    return (long long)page * page_elems + ((long long)((layer * Hk + g) * 2 + kv) * kPageTokens + (pos & 63)) * d;
  }
  __device__ __forceinline__ const bf16* Block(int slot, int block, int layer, int g, int kv) const {
    const int page = block_table[slot * max_blocks + block];
    if (page < 0) {
      atomicCAS(&g_shahd_device_error, 0, kDevErrNoPage);
      return nullptr;
    }
    return pool + (size_t)page * page_elems + (size_t)((layer * Hk + g) * 2 + kv) * kPageTokens * d;
  }
};

// ---- epilogues: apply(m, n, v0, v1) gets the fp32 dot products of output columns n and n+1 (n even)
// of row m. Pairs keep RoPE's interleaved (2i, 2i+1) rotation (RotaryEmbedding.ts:42-60) and the
// gate/up columns of the interleaved W1|W3 layout in one thread.

// Q/K/V projection: RoPE on q and k at the row's position, q to fp32 scratch, k/v appended to the cache.
struct EpiQKV {
  float* q;          // [M, H*d]
  KvView kv;
  int layer;
  const int* pos;    // [M]
  const int* slot;   // [M]
  const float* rope_cos;  // [C, d/2] or nullptr (learned positions)
  const float* rope_sin;
  int H, Hk, d;
  __device__ __forceinline__ void apply(int m, int n, float v0, float v1, int N) const {
    const int hd = H * d;
    const int j = n % d;  // even: d is even and n is even
    const int p = pos[m];
    if (n < hd + Hk * d && rope_cos != nullptr) {
      const float c = rope_cos[p * (d >> 1) + (j >> 1)], s = rope_sin[p * (d >> 1) + (j >> 1)];
      const float r0 = v0 * c - v1 * s, r1 = v0 * s + v1 * c;
      v0 = r0;
      v1 = r1;
    }
    if (n < hd) {
      *reinterpret_cast<float2*>(q + (size_t)m * hd + n) = make_float2(v0, v1);
      return;
    }
    const int kvsel = n < hd + Hk * d ? 0 : 1;
    const int g = (n - hd - kvsel * Hk * d) / d;
    const long long off = kv.Offset(slot[m], p, layer, g, kvsel);
    if (off < 0) return;
    *reinterpret_cast<__nv_bfloat162*>(kv.pool + off + j) = __floats2bfloat162_rn(v0, v1);
  }
};

// Residual update x += v (+ bias): the attention output projection (summed per-head Wo,
// CachedForward.ts:75-84) and the MLP down projection (CachedForward.ts:86-87).
struct EpiResid {
  float* x;  // [M, ldx]
  int ldx;
  const float* bias;  // nullable
  __device__ __forceinline__ void apply(int m, int n, float v0, float v1, int N) const {
    float* p = x + (size_t)m * ldx + n;
    if (bias) {
      v0 += bias[n];
      if (n + 1 < N) v1 += bias[n + 1];
    }
    p[0] += v0;
    if (n + 1 < N) p[1] += v1;
  }
};

// Gated MLP hidden: act[j] = Act(x·W1[:,j]) * (x·W3[:,j]) with W1/W3 interleaved per column pair
// (MlpRow, CachedRowMath.ts:107-112; SiluValue Silu.ts:8-10; GeluValue Gelu.ts:7-14).
struct EpiGated {
  float* act;  // [M, F]
  int F;
  int gelu;
  __device__ __forceinline__ void apply(int m, int n, float g, float u, int N) const {
    float a;
    if (gelu) {
      const float c = 0.7978845608028654f;  // sqrt(2/pi)
      a = 0.5f * g * (1.0f + tanhf(c * (g + 0.044715f * g * g * g)));
    } else {
      a = g * (1.0f / (1.0f + __expf(-g)));
    }
    act[(size_t)m * F + (n >> 1)] = a * u;
  }
};

// Relu MLP hidden: relu(x·Wfc + bfc) (MlpRow, CachedRowMath.ts:95-101).
struct EpiReluFc {
  float* act;  // [M, F]
  int F;
  const float* bias;
  __device__ __forceinline__ void apply(int m, int n, float v0, float v1, int N) const {
    float* p = act + (size_t)m * F + n;
    v0 += bias[n];
    p[0] = v0 > 0.f ? v0 : 0.f;
    if (n + 1 < N) {
      v1 += bias[n + 1];
      p[1] = v1 > 0.f ? v1 : 0.f;
    }
  }
};

// LM head: logits = xf·Wteᵀ + bias (HeadLogitsRow, CachedRowMath.ts:117-137); also feeds argmax.
struct EpiLogits {
  float* logits;      // [M, V] or nullptr
  const float* bias;  // [V]
  __device__ __forceinline__ void apply(int m, int n, float& v0, float& v1, int N) const {
    v0 += bias[n];
    if (n + 1 < N) v1 += bias[n + 1];
    if (logits) {
      float* p = logits + (size_t)m * N + n;
      p[0] = v0;
      if (n + 1 < N) p[1] = v1;
    }
  }
};

template <class Epi>
struct IsLogits {
  static constexpr bool value = false;
};
template <>
struct IsLogits<EpiLogits> {
  static constexpr bool value = true;
};

// ---- SIMT linear (GEMV regime, few rows): out[m, n] = sum_k T(a[m, k]) * W[n, k] --------------------
// T is the row norm of the layer (NormRow, CachedRowMath.ts:25-56) or identity. W is bf16 [N, Kp]
// (K padded to a multiple of 8 with zeros). 4 warps x 2 columns per CTA; rows in tiles of MT.

struct LinearArgs {
  const float* a;
  int lda;
  int M;
  int K;   // logical reduction length
  int Kp;  // padded row length of W (multiple of 8)
  const bf16* w;
  int N;
  const float* gamma;
  const float* beta;
  float eps;
  float* am_val;  // argmax partials [M, gridDim.x] (logits only)
  int* am_idx;
};

constexpr int kSimtWarps = 4;
constexpr int kSimtCols = kSimtWarps * 2;

template <int MT, int NORM>
__device__ __forceinline__ void StageRowsNormalized(const LinearArgs& la, float* sA, int m0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < MT; r += kSimtWarps) {
    float* dst = sA + (size_t)r * la.Kp;
    if (m0 + r >= la.M) {
      for (int k = lane; k < la.Kp; k += 32) dst[k] = 0.f;
      continue;
    }
    const float* src = la.a + (size_t)(m0 + r) * la.lda;
    float mu = 0.f, is = 1.f;
    if (NORM == kNormRms) {
      float ss = 0.f;
      for (int k = lane; k < la.K; k += 32) ss += src[k] * src[k];
      ss = WarpSum(ss);
      is = 1.0f / sqrtf(ss / la.K + la.eps);
    } else if (NORM == kNormLayer) {
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
    for (int k = lane; k < la.Kp; k += 32) {
      float v = 0.f;
      if (k < la.K) {
        v = src[k];
        if (NORM == kNormRms) v = la.gamma[k] * v * is;
        else if (NORM == kNormLayer) v = la.gamma[k] * ((v - mu) * is) + la.beta[k];
      }
      dst[k] = v;
    }
  }
}

template <int MT, int NORM, class Epi>
__global__ void __launch_bounds__(kSimtWarps * 32) LinearSimtKernel(LinearArgs la, Epi epi) {
  extern __shared__ __align__(16) float sA[];  // [MT][Kp]
  __shared__ float s_am_v[kSimtWarps][MT];
  __shared__ int s_am_i[kSimtWarps][MT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MT;
  StageRowsNormalized<MT, NORM>(la, sA, m0);
  __syncthreads();

  const int col = (blockIdx.x * kSimtWarps + warp) * 2;
  float acc[MT][2];
#pragma unroll
  for (int m = 0; m < MT; m++) acc[m][0] = acc[m][1] = 0.f;
  if (col < la.N) {
    const bf16* w0 = la.w + (size_t)col * la.Kp;
    const bool has1 = col + 1 < la.N;
    const bf16* w1 = has1 ? w0 + la.Kp : w0;
    for (int k = lane * 8; k < la.Kp; k += 256) {
      uint4 u0 = LoadNc16(w0 + k);
      uint4 u1 = LoadNc16(w1 + k);
      float f0[8], f1[8];
      Bf16x8ToFloat(u0, f0);
      Bf16x8ToFloat(u1, f1);
#pragma unroll
      for (int m = 0; m < MT; m++) {
        const float4 x0 = *reinterpret_cast<const float4*>(sA + (size_t)m * la.Kp + k);
        const float4 x1 = *reinterpret_cast<const float4*>(sA + (size_t)m * la.Kp + k + 4);
        const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int j = 0; j < 8; j++) {
          acc[m][0] = fmaf(xs[j], f0[j], acc[m][0]);
          acc[m][1] = fmaf(xs[j], f1[j], acc[m][1]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; m++) {
    acc[m][0] = WarpSum(acc[m][0]);
    acc[m][1] = WarpSum(acc[m][1]);
  }
  float bv = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll
  for (int m = 0; m < MT; m++) {
    if (lane == m && m0 + m < la.M && col < la.N) {
      float v0 = acc[m][0], v1 = acc[m][1];
      epi.apply(m0 + m, col, v0, v1, la.N);
      if constexpr (IsLogits<Epi>::value) {
        ArgmaxMerge(bv, bi, v0, col);
        if (col + 1 < la.N) ArgmaxMerge(bv, bi, v1, col + 1);
      }
    }
  }
  if constexpr (IsLogits<Epi>::value) {
    if (lane < MT) {
      s_am_v[warp][lane] = bv;
      s_am_i[warp][lane] = bi;
    }
    __syncthreads();
    if (threadIdx.x < MT && m0 + threadIdx.x < la.M) {
      float v = -INFINITY;
      int i = 0x7fffffff;
      for (int w = 0; w < kSimtWarps; w++) ArgmaxMerge(v, i, s_am_v[w][threadIdx.x], s_am_i[w][threadIdx.x]);
      la.am_val[(size_t)(m0 + threadIdx.x) * gridDim.x + blockIdx.x] = v;
      la.am_idx[(size_t)(m0 + threadIdx.x) * gridDim.x + blockIdx.x] = i;
    }
  }
}

// ---- embedding: x = Wte[token] (+ Wpe[pos]) (AdvanceOneToken, CachedForward.ts:48-53) ---------------

struct EmbedArgs {
  const int* slot;      // [M]
  const int* tok;       // direct tokens [M] (when poff == nullptr)
  const int* prompt;    // packed prompt ids (prefill gather)
  const int* poff;      // [M] offset of each row's context in `prompt`, or nullptr
  const int* seq_len;   // [slots]
  int* pos;             // [M] out: the row's position
  const float* wte;     // [V, E]
  const float* wpe;     // [C, E] or nullptr
  float* x;             // [M, E]
  int E;
};

__global__ void EmbedKernel(EmbedArgs e) {
  const int r = blockIdx.x;
  const int p = e.seq_len[e.slot[r]];
  const int tok = e.poff ? e.prompt[e.poff[r] + p] : e.tok[r];
  if (threadIdx.x == 0) e.pos[r] = p;
  const float* src = e.wte + (size_t)tok * e.E;
  const float* pe = e.wpe ? e.wpe + (size_t)p * e.E : nullptr;
  float* dst = e.x + (size_t)r * e.E;
  for (int j = threadIdx.x; j < e.E; j += blockDim.x) dst[j] = pe ? src[j] + pe[j] : src[j];
}

// ---- decode attention over the paged cache (AttendRow, CachedRowMath.ts:60-86) ---------------------
// Grid (chunk, kv head, row). Each CTA takes one 64-position page of one KV head for one row, scores it
// against the head's whole query group (GQA: heads g*G .. g*G+G-1 share the page), and writes a
// partial (o, max, sum). The last CTA of a (row, kv head) to finish — counted with an atomic — merges
// the partials in chunk order; with a single chunk the CTA writes the context directly.

struct AttnArgs {
  const float* q;   // [M, H*d] post-RoPE
  float* ctx;       // [M, H*d]
  KvView kv;
  int layer;
  const int* pos;
  const int* slot;
  int H, Hk, G, d;
  float scale;
  int max_chunks;
  float* part_o;    // [M, H, max_chunks, d]
  float* part_m;    // [M, H, max_chunks]
  float* part_l;
  int* counter;     // [M, Hk], zero between launches
};

constexpr int kAttnThreads = 128;
constexpr int kMaxGroup = 8;

__device__ __forceinline__ void AttnMerge(const AttnArgs& aa, int m, int g, int nch) {
  const int hd = aa.H * aa.d;
  for (int e = threadIdx.x; e < aa.G * aa.d; e += blockDim.x) {
    const int i = e / aa.d, j = e % aa.d;
    const int h = g * aa.G + i;
    const size_t base = ((size_t)m * aa.H + h) * aa.max_chunks;
    float mx = -INFINITY;
    for (int c = 0; c < nch; c++) mx = fmaxf(mx, __ldcg(aa.part_m + base + c));
    float num = 0.f, den = 0.f;
    for (int c = 0; c < nch; c++) {
      const float w = __expf(__ldcg(aa.part_m + base + c) - mx);
      num += w * __ldcg(aa.part_o + (base + c) * aa.d + j);
      den += w * __ldcg(aa.part_l + base + c);
    }
    aa.ctx[(size_t)m * hd + h * aa.d + j] = num / den;
  }
}

// Writes this CTA's per-head results; merges when it is the last chunk of its (row, kv head).
__device__ __forceinline__ void AttnFinishChunk(const AttnArgs& aa, int m, int g, int c, int nch, const float* so,
                                                const float* sm, const float* sl) {
  const int hd = aa.H * aa.d;
  if (nch == 1) {
    for (int e = threadIdx.x; e < aa.G * aa.d; e += blockDim.x) {
      const int i = e / aa.d, j = e % aa.d;
      aa.ctx[(size_t)m * hd + (g * aa.G + i) * aa.d + j] = so[e] / sl[i];
    }
    return;
  }
  for (int e = threadIdx.x; e < aa.G * aa.d; e += blockDim.x) {
    const int i = e / aa.d, j = e % aa.d;
    const size_t base = ((size_t)m * aa.H + g * aa.G + i) * aa.max_chunks + c;
    aa.part_o[base * aa.d + j] = so[e];
    if (j == 0) {
      aa.part_m[base] = sm[i];
      aa.part_l[base] = sl[i];
    }
  }
  __threadfence();
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(aa.counter + m * aa.Hk + g, 1);
    s_last = (prev == nch - 1);
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    AttnMerge(aa, m, g, nch);
    if (threadIdx.x == 0) aa.counter[m * aa.Hk + g] = 0;
  }
}

// Fast path: head_dim D (multiple of 8, 32..128) known at compile time.
template <int D>
__global__ void __launch_bounds__(kAttnThreads) AttnDecodeKernel(AttnArgs aa) {
  constexpr int LPP = D / 8;           // lanes per position (16 B of K each)
  constexpr int PPW = 32 / LPP;        // positions per warp pass
  constexpr int JPL = D / 32;          // output dims per lane
  __shared__ float sq[kMaxGroup][D];
  __shared__ float ss[kMaxGroup][kPageTokens];
  __shared__ float so_part[kAttnThreads / 32][kMaxGroup * D];
  __shared__ float so[kMaxGroup * D];
  __shared__ float sm[kMaxGroup], sl[kMaxGroup];
  const int c = blockIdx.x, g = blockIdx.y, m = blockIdx.z;
  const int p = aa.pos[m];
  const int nch = (p + kPageTokens) / kPageTokens;  // positions 0..p
  if (c >= nch) return;
  const int t0 = c * kPageTokens;
  const int tn = min(kPageTokens, p + 1 - t0);
  const int G = aa.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = aa.H * D;
  const int slot = aa.slot[m];
  const bf16* kb = aa.kv.Block(slot, c, aa.layer, g, 0);
  const bf16* vb = aa.kv.Block(slot, c, aa.layer, g, 1);
  const int tv = kb ? tn : 0;  // a missing page (recorded as an error) contributes no positions

  for (int e = threadIdx.x; e < G * D; e += blockDim.x) sq[e / D][e % D] = aa.q[(size_t)m * hd + g * G * D + e];
  __syncthreads();

  // scores s[i][t] = (q_i · k_t) * scale
  const int seg = lane % LPP;
  for (int tb = warp * PPW; tb < kPageTokens; tb += (kAttnThreads / 32) * PPW) {
    const int t = tb + lane / LPP;
    float kf[8];
    if (t < tv) {
      uint4 u = LoadNc16(kb + (size_t)t * D + seg * 8);
      Bf16x8ToFloat(u, kf);
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) kf[j] = 0.f;
    }
    for (int i = 0; i < G; i++) {
      float part = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) part = fmaf(kf[j], sq[i][seg * 8 + j], part);
#pragma unroll
      for (int o = LPP / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (seg == 0 && t < tv) ss[i][t] = part * aa.scale;
    }
  }
  __syncthreads();

  // per-head max and exp-sum over this chunk
  for (int i = warp; i < G; i += kAttnThreads / 32) {
    float mx = -INFINITY;
    for (int t = lane; t < tv; t += 32) mx = fmaxf(mx, ss[i][t]);
    mx = WarpMax(mx);
    float sum = 0.f;
    for (int t = lane; t < tv; t += 32) {
      const float e = __expf(ss[i][t] - mx);
      ss[i][t] = e;
      sum += e;
    }
    sum = WarpSum(sum);
    if (lane == 0) {
      sm[i] = mx;
      sl[i] = sum;
    }
  }
  __syncthreads();

  // o[i][j] = sum_t e[i][t] * v_t[j]; warps split t, lanes split j
  float o[kMaxGroup][JPL];
#pragma unroll
  for (int i = 0; i < kMaxGroup; i++)
#pragma unroll
    for (int jj = 0; jj < JPL; jj++) o[i][jj] = 0.f;
  for (int t = warp; t < tv; t += kAttnThreads / 32) {
    float vf[JPL];
    if constexpr (JPL == 2) {
      const float2 v2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vb + (size_t)t * D + lane * 2));
      vf[0] = v2.x;
      vf[1] = v2.y;
    } else {
#pragma unroll
      for (int jj = 0; jj < JPL; jj++) vf[jj] = __bfloat162float(vb[(size_t)t * D + lane * JPL + jj]);
    }
#pragma unroll
    for (int i = 0; i < kMaxGroup; i++) {
      if (i < G) {
        const float e = ss[i][t];
#pragma unroll
        for (int jj = 0; jj < JPL; jj++) o[i][jj] = fmaf(e, vf[jj], o[i][jj]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxGroup; i++)
    if (i < G)
#pragma unroll
      for (int jj = 0; jj < JPL; jj++) so_part[warp][i * D + lane * JPL + jj] = o[i][jj];
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnThreads / 32; w++) s += so_part[w][e];
    so[e] = s;
  }
  __syncthreads();
  AttnFinishChunk(aa, m, g, c, nch, so, sm, sl);
}

// Any even head_dim up to 128 (the reference's small test shapes use d = 4, 8, 16): scalar loops.
constexpr int kMaxHeadDimGeneric = 128;
__global__ void __launch_bounds__(kAttnThreads) AttnDecodeGenericKernel(AttnArgs aa) {
  __shared__ float sq[kMaxGroup * kMaxHeadDimGeneric];
  __shared__ float ss[kMaxGroup][kPageTokens];
  __shared__ float so[kMaxGroup * kMaxHeadDimGeneric];
  __shared__ float sm[kMaxGroup], sl[kMaxGroup];
  const int c = blockIdx.x, g = blockIdx.y, m = blockIdx.z;
  const int p = aa.pos[m];
  const int nch = (p + kPageTokens) / kPageTokens;
  if (c >= nch) return;
  const int t0 = c * kPageTokens;
  const int tn = min(kPageTokens, p + 1 - t0);
  const int G = aa.G, D = aa.d;
  const int hd = aa.H * D;
  const int slot = aa.slot[m];
  const bf16* kb = aa.kv.Block(slot, c, aa.layer, g, 0);
  const bf16* vb = aa.kv.Block(slot, c, aa.layer, g, 1);
  const int tv = kb ? tn : 0;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) sq[e] = aa.q[(size_t)m * hd + g * G * D + e];
  __syncthreads();
  for (int e = threadIdx.x; e < G * kPageTokens; e += blockDim.x) {
    const int i = e / kPageTokens, t = e % kPageTokens;
    if (t < tv) {
      float dot = 0.f;
      for (int j = 0; j < D; j++) dot = fmaf(sq[i * D + j], __bfloat162float(kb[(size_t)t * D + j]), dot);
      ss[i][t] = dot * aa.scale;
    }
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int i = threadIdx.x;
    float mx = -INFINITY;
    for (int t = 0; t < tv; t++) mx = fmaxf(mx, ss[i][t]);
    float sum = 0.f;
    for (int t = 0; t < tv; t++) {
      const float e = __expf(ss[i][t] - mx);
      ss[i][t] = e;
      sum += e;
    }
    sm[i] = mx;
    sl[i] = sum;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int i = e / D, j = e % D;
    float acc = 0.f;
    for (int t = 0; t < tv; t++) acc = fmaf(ss[i][t], __bfloat162float(vb[(size_t)t * D + j]), acc);
    so[e] = acc;
  }
  __syncthreads();
  AttnFinishChunk(aa, m, g, c, nch, so, sm, sl);
}

// ---- finish: positions advance; greedy argmax over the head's per-CTA partials -------------------------

struct FinishArgs {
  int M;
  const int* slot;
  const int* pos;
  int* seq_len;
  const float* am_val;  // [M, nblk] or nullptr (no head this step)
  const int* am_idx;
  int nblk;
  int* next_ids;    // [M] or nullptr
  int* cur_tok;     // [M] or nullptr: next input token of the decode loop
  int* out_ids;     // [M, out_ld] or nullptr
  int out_ld;
  int* gen_count;   // [M]
  const int* sampled;  // [M] ids chosen by the sampler (stochastic decoding), or nullptr for greedy
};

__global__ void FinishKernel(FinishArgs f) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= f.M) return;
  f.seq_len[f.slot[r]] = f.pos[r] + 1;
  if (f.am_val == nullptr && f.sampled == nullptr) return;
  int id;
  if (f.sampled) {
    id = f.sampled[r];
  } else {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int b = 0; b < f.nblk; b++) ArgmaxMerge(bv, bi, f.am_val[(size_t)r * f.nblk + b], f.am_idx[(size_t)r * f.nblk + b]);
    id = bi == 0x7fffffff ? 0 : bi;
  }
  if (f.next_ids) f.next_ids[r] = id;
  if (f.cur_tok) f.cur_tok[r] = id;
  if (f.out_ids) {
    const int k = f.gen_count[r];
    f.out_ids[(size_t)r * f.out_ld + k] = id;
    f.gen_count[r] = k + 1;
  }
}

}  // namespace shahd
