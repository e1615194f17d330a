// Decode-step kernels for one batched cached step over M rows (row r = one sequence's next token).
// Restates AdvanceOneToken + HeadLogitsRow (Brain/Sampling/CachedForward.ts:32-96,
// CachedRowMath.ts:14-137) as: embed -> per layer [norm+QKV+RoPE+KV append] -> [attention over the
// paged cache] -> [O projection + residual] -> [norm + gate/up + SwiGLU/GeGLU | fc + ReLU] ->
// [down projection + residual] -> [final norm + LM head + argmax partials] -> finish.
//
// Norms are folded into the projection that consumes them: the weights carry gamma (W' = W·diag(gamma),
// repacked once), and the kernel applies the row statistics: RMSNorm out = is·(x·W'), LayerNorm
// out = is·(x·W' - mu·c1) + c2 with c1 = sum_k W', c2 = beta·W (NormRow, CachedRowMath.ts:25-56).
// Activations keep an fp32 master copy (read by the CUDA-core kernels) and a bf16 copy (the tensor-core
// operand, loaded by TMA).
#pragma once

#include "common.cuh"

namespace shahd {

__device__ int g_shahd_device_error;  // 0 = ok; otherwise the first kDevErr* code recorded
constexpr int kDevErrUmmaTimeout = 1;
constexpr int kDevErrGemmTimeout = 2;
constexpr int kDevErrNoPage = 3;
constexpr int kDevErrAttnTimeout = 4;

constexpr uint32_t kWaitLimit = 1u << 22;  // mbarrier probes before a wait gives up

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

__device__ __forceinline__ void StoreBf16x2(bf16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

// 16 consecutive floats / bf16 to and from memory in 16-byte pieces (callers check alignment).
__device__ __forceinline__ void Load16f(const float* p, float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float4 t = reinterpret_cast<const float4*>(p)[i];
    v[4 * i] = t.x;
    v[4 * i + 1] = t.y;
    v[4 * i + 2] = t.z;
    v[4 * i + 3] = t.w;
  }
}
template <int N>
__device__ __forceinline__ void StoreNf(float* p, const float* v) {
#pragma unroll
  for (int i = 0; i < N / 4; i++)
    reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}
template <int N>
__device__ __forceinline__ void StoreNbf(bf16* p, const float* v) {
#pragma unroll
  for (int i = 0; i < N / 8; i++) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    reinterpret_cast<uint4*>(p)[i] = u;
  }
}

// ---- epilogues: apply(m, n, v0, v1) gets the final values of output columns n and n+1 (n even) of row
// m (norm already applied). Pairs keep RoPE's interleaved (2i, 2i+1) rotation (RotaryEmbedding.ts:42-60)
// and the gate/up columns of the interleaved W1|W3 layout in one thread.
//
// The tensor-core kernel also has a 16-column form for a chunk n..n+15 (n a multiple of 16) when
// vec_ok(N): load16 issues every global read the chunk needs (residual, bias, RoPE table, KV page lookup)
// and can run before the accumulator is ready; store16 then only computes and writes, with 16-byte
// stores. Reads never depend on this launch's own writes, so no load waits behind a store.

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
    StoreBf16x2(kv.pool + off + j, v0, v1);
  }
  struct Pre {
    float c[8], s[8];
    float* qdst;  // q row chunk, or nullptr for k/v
    bf16* kvdst;  // KV page row chunk, or nullptr (q, or no page)
  };
  __device__ __forceinline__ bool vec_ok(int N) const { return d % 16 == 0 && (H * d) % 4 == 0; }
  __device__ __forceinline__ Pre load16(int m, int n) const {
    Pre pr;
    const int hd = H * d, j = n % d, p = pos[m];
    const bool rope = n < hd + Hk * d && rope_cos != nullptr;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      pr.c[i] = 1.f;
      pr.s[i] = 0.f;
    }
    if (rope) {
      const float* cp = rope_cos + p * (d >> 1) + (j >> 1);
      const float* sp = rope_sin + p * (d >> 1) + (j >> 1);
#pragma unroll
      for (int i = 0; i < 2; i++) {
        const float4 c4 = reinterpret_cast<const float4*>(cp)[i], s4 = reinterpret_cast<const float4*>(sp)[i];
        pr.c[4 * i] = c4.x; pr.c[4 * i + 1] = c4.y; pr.c[4 * i + 2] = c4.z; pr.c[4 * i + 3] = c4.w;
        pr.s[4 * i] = s4.x; pr.s[4 * i + 1] = s4.y; pr.s[4 * i + 2] = s4.z; pr.s[4 * i + 3] = s4.w;
      }
    }
    pr.qdst = nullptr;
    pr.kvdst = nullptr;
    if (n < hd) {
      pr.qdst = q + (size_t)m * hd + n;
    } else {
      const int kvsel = n < hd + Hk * d ? 0 : 1;
      const int g = (n - hd - kvsel * Hk * d) / d;
      const long long off = kv.Offset(slot[m], p, layer, g, kvsel);
      if (off >= 0) pr.kvdst = kv.pool + off + j;
    }
    return pr;
  }
  __device__ __forceinline__ void store16(int m, int n, float (&v)[16], const Pre& pr) const {
#pragma unroll
    for (int i = 0; i < 8; i++) {  // identity rotation (c = 1, s = 0) where RoPE does not apply
      const float a = v[2 * i], b = v[2 * i + 1];
      v[2 * i] = a * pr.c[i] - b * pr.s[i];
      v[2 * i + 1] = a * pr.s[i] + b * pr.c[i];
    }
    if (pr.qdst) StoreNf<16>(pr.qdst, v);
    else if (pr.kvdst) StoreNbf<16>(pr.kvdst, v);
  }
};

// Residual update x += v (+ bias), bf16 copy refreshed: the attention output projection (summed
// per-head Wo, CachedForward.ts:75-84) and the MLP down projection (CachedForward.ts:86-87).
struct EpiResid {
  float* x;  // [M, ldx]
  bf16* xb;  // [M, ldxb]
  int ldx, ldxb;
  const float* bias;  // nullable
  __device__ __forceinline__ void apply(int m, int n, float v0, float v1, int N) const {
    float* p = x + (size_t)m * ldx + n;
    if (bias) {
      v0 += bias[n];
      if (n + 1 < N) v1 += bias[n + 1];
    }
    const float a = p[0] + v0;
    p[0] = a;
    float b = 0.f;
    if (n + 1 < N) {
      b = p[1] + v1;
      p[1] = b;
    }
    StoreBf16x2(xb + (size_t)m * ldxb + n, a, b);
  }
  struct Pre {
    float x[16];  // residual (+ bias)
  };
  __device__ __forceinline__ bool vec_ok(int N) const { return ldx % 4 == 0 && ldxb % 8 == 0; }
  __device__ __forceinline__ Pre load16(int m, int n) const {
    Pre pr;
    Load16f(x + (size_t)m * ldx + n, pr.x);
    if (bias) {
      float b[16];
      Load16f(bias + n, b);
#pragma unroll
      for (int i = 0; i < 16; i++) pr.x[i] += b[i];
    }
    return pr;
  }
  __device__ __forceinline__ void store16(int m, int n, float (&v)[16], const Pre& pr) const {
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] += pr.x[i];
    StoreNf<16>(x + (size_t)m * ldx + n, v);
    StoreNbf<16>(xb + (size_t)m * ldxb + n, v);
  }
};

// The gate activations (SiluValue, Silu.ts:8-10: g / (1 + e^-g); GeluValue, Gelu.ts:7-14: the tanh form
// 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3)))) with tanh(u) = 1 - 2 / (1 + e^(2u)), from __expf and the
// approximate divide (a few ulp, far below the bf16 rounding of the result); both saturate correctly (an
// infinite exponential gives a zero quotient).
__device__ __forceinline__ float GateAct(float g, int gelu) {
  if (gelu) {
    const float u = 0.7978845608028654f * (g + 0.044715f * g * g * g);  // sqrt(2/pi) (g + 0.044715 g^3)
    return 0.5f * g * (2.0f - __fdividef(2.0f, 1.0f + __expf(2.0f * u)));
  }
  return __fdividef(g, 1.0f + __expf(-g));
}

// Gated MLP hidden: act[j] = Act(x·W1[:,j]) * (x·W3[:,j]) with W1/W3 interleaved per column pair
// (MlpRow, CachedRowMath.ts:107-112; SiluValue Silu.ts:8-10; GeluValue Gelu.ts:7-14).
struct EpiGated {
  float* act;  // [M, F], or nullptr when only the bf16 copy is read (tensor-core down projection)
  bf16* actb;  // [M, ldb]
  int F, ldb;
  int gelu;
  __device__ __forceinline__ void apply(int m, int n, float g, float u, int N) const {
    const float h = GateAct(g, gelu) * u;
    if (act) act[(size_t)m * F + (n >> 1)] = h;
    actb[(size_t)m * ldb + (n >> 1)] = __float2bfloat16_rn(h);
  }
  struct Pre {};
  __device__ __forceinline__ bool vec_ok(int N) const { return F % 4 == 0 && ldb % 8 == 0; }
  __device__ __forceinline__ Pre load16(int, int) const { return Pre{}; }
  __device__ __forceinline__ void store16(int m, int n, float (&v)[16], const Pre&) const {
    float h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      h[i] = GateAct(v[2 * i], gelu) * v[2 * i + 1];
    }
    if (act) StoreNf<8>(act + (size_t)m * F + (n >> 1), h);
    StoreNbf<8>(actb + (size_t)m * ldb + (n >> 1), h);
  }
};

// Relu MLP hidden: relu(x·Wfc + bfc) (MlpRow, CachedRowMath.ts:95-101).
struct EpiReluFc {
  float* act;  // [M, F]
  bf16* actb;
  int F, ldb;
  const float* bias;
  __device__ __forceinline__ void apply(int m, int n, float v0, float v1, int N) const {
    float* p = act + (size_t)m * F + n;
    v0 += bias[n];
    v0 = v0 > 0.f ? v0 : 0.f;
    p[0] = v0;
    if (n + 1 < N) {
      v1 += bias[n + 1];
      v1 = v1 > 0.f ? v1 : 0.f;
      p[1] = v1;
    } else {
      v1 = 0.f;
    }
    StoreBf16x2(actb + (size_t)m * ldb + n, v0, v1);
  }
  struct Pre {
    float b[16];
  };
  __device__ __forceinline__ bool vec_ok(int N) const { return F % 4 == 0 && ldb % 8 == 0; }
  __device__ __forceinline__ Pre load16(int, int n) const {
    Pre pr;
    Load16f(bias + n, pr.b);
    return pr;
  }
  __device__ __forceinline__ void store16(int m, int n, float (&v)[16], const Pre& pr) const {
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float t = v[i] + pr.b[i];
      v[i] = t > 0.f ? t : 0.f;
    }
    StoreNf<16>(act + (size_t)m * F + n, v);
    StoreNbf<16>(actb + (size_t)m * ldb + n, v);
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
  int V;  // row stride of logits (= N of the head launch)
  struct Pre {
    float b[16];
  };
  __device__ __forceinline__ bool vec_ok(int N) const { return N % 4 == 0; }
  __device__ __forceinline__ Pre load16(int, int n) const {
    Pre pr;
    Load16f(bias + n, pr.b);
    return pr;
  }
  // adds the bias in place, so the caller's argmax sees the final logits
  __device__ __forceinline__ void store16(int m, int n, float (&v)[16], const Pre& pr) const {
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] += pr.b[i];
    if (logits) StoreNf<16>(logits + (size_t)m * V + n, v);
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

// ---- projection arguments ------------------------------------------------------------------------

struct LinearArgs {
  const float* a;   // fp32 rows [M, lda]  (CUDA-core path)
  int lda;
  const bf16* ab;   // bf16 rows [a_rows, ldab] (tensor-core path, TMA)
  int ldab;
  int a_rows;
  int M;
  int K;            // logical reduction length
  int Kp;           // padded row length of W and ab (multiple of 8)
  const bf16* w;    // [N, Kp], gamma folded in for norm-consuming projections
  int N;
  float eps;
  const float* c1;  // LayerNorm: sum_k W'[n,k]
  const float* c2;  // LayerNorm: sum_k beta[k] W[n,k]
  float* am_val;    // argmax partials [M, gridDim.x] (logits only)
  int* am_idx;
  float* ws;        // split-K partial tiles (tensor-core path, no norm), or nullptr: no split
  int* ws_cnt;      // [N tiles] arrival counters, zero between launches
  int kcluster;     // the split-K CTAs of a tile form a cluster and sum their partials in shared memory
  const float* stats;  // [M][2] norm statistics (mean, 1/std) of the rows (persistent prefill kernel), or nullptr
};

// ---- SIMT linear (GEMV regime, few rows): out[m, n] = sum_k xhat[m, k] * W'[n, k] -------------------
// xhat = x·is (RMS) or (x - mu)·is (LayerNorm, + c2 in the epilogue) or x. 4 warps x 2 columns per CTA.

constexpr int kSimtWarps = 4;
constexpr int kSimtCols = kSimtWarps * 2;

template <int MT, int NORM>
__device__ __forceinline__ void StageRowsNormalized(const LinearArgs& la, float* sA, int m0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < MT; r += kSimtWarps) {
    float* dst = sA + (size_t)r * la.Kp;
    if (m0 + r >= la.M) {
      for (int k = lane * 4; k < la.Kp; k += 128) *reinterpret_cast<float4*>(dst + k) = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    const float* src = la.a + (size_t)(m0 + r) * la.lda;
    // copy (zero-padded) into shared memory first; the statistics are then taken from there
    const bool vec = (la.lda & 3) == 0 && (la.K & 3) == 0;
#pragma unroll 4
    for (int k = lane * 4; k < la.Kp; k += 128) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (vec && k < la.K) {
        v = *reinterpret_cast<const float4*>(src + k);
      } else if (!vec) {
        if (k < la.K) v.x = src[k];
        if (k + 1 < la.K) v.y = src[k + 1];
        if (k + 2 < la.K) v.z = src[k + 2];
        if (k + 3 < la.K) v.w = src[k + 3];
      }
      *reinterpret_cast<float4*>(dst + k) = v;
    }
    if (NORM == kNormNone) continue;
    __syncwarp();
    float mu = 0.f, is;
    if (NORM == kNormRms) {
      float ss = 0.f;
      for (int k = lane; k < la.K; k += 32) ss += dst[k] * dst[k];
      ss = WarpSum(ss);
      is = 1.0f / sqrtf(ss / la.K + la.eps);
    } else {
      float s = 0.f;
      for (int k = lane; k < la.K; k += 32) s += dst[k];
      mu = WarpSum(s) / la.K;
      float v = 0.f;
      for (int k = lane; k < la.K; k += 32) {
        const float t = dst[k] - mu;
        v += t * t;
      }
      v = WarpSum(v) / la.K;
      is = 1.0f / sqrtf(v + la.eps);
    }
    for (int k = lane; k < la.K; k += 32) dst[k] = (dst[k] - mu) * is;
  }
}

template <int MT, int NORM, class Epi>
__global__ void __launch_bounds__(kSimtWarps * 32) LinearSimtKernel(LinearArgs la, Epi epi) {
  extern __shared__ __align__(16) float sA[];  // [MT][Kp]
  __shared__ float s_am_v[kSimtWarps][MT];
  __shared__ int s_am_i[kSimtWarps][MT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * MT;
  GridDepWait();
  GridDepLaunch();
  StageRowsNormalized<MT, NORM>(la, sA, m0);
  __syncthreads();

  const int col = (blockIdx.x * kSimtWarps + warp) * 2;
  float acc[MT][2];
#pragma unroll
  for (int m = 0; m < MT; m++) acc[m][0] = acc[m][1] = 0.f;
  if (col < la.N) {
    const bf16* w0 = la.w + (size_t)col * la.Kp;
    const bf16* w1 = col + 1 < la.N ? w0 + la.Kp : w0;
#pragma unroll 4
    for (int k = lane * 8; k < la.Kp; k += 256) {
      const uint4 u0 = LoadNc16(w0 + k);
      const uint4 u1 = LoadNc16(w1 + k);
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
      if (NORM == kNormLayer) {
        v0 += la.c2[col];
        if (col + 1 < la.N) v1 += la.c2[col + 1];
      }
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
  const int* pos_in;    // [M] explicit positions (batched prefill rows), or nullptr: the slot's length
  const int* slot;      // [M]
  const int* tok;       // direct tokens [M] (when poff == nullptr)
  const int* prompt;    // packed prompt ids (prefill gather)
  const int* poff;      // [M] offset of each row's context in `prompt`, or nullptr
  const int* seq_len;   // [slots]
  int* pos;             // [M] out: the row's position
  const float* wte;     // [V, E]
  const float* wpe;     // [C, E] or nullptr
  float* x;             // [M, E]
  bf16* xb;             // [M, ldxb]
  int E, ldxb;
};

__global__ void EmbedKernel(EmbedArgs e) {
  GridDepWait();
  GridDepLaunch();
  const int r = blockIdx.x;
  const int p = e.pos_in ? e.pos_in[r] : e.seq_len[e.slot[r]];
  const int tok = e.poff ? e.prompt[e.poff[r] + p] : e.tok[r];
  if (threadIdx.x == 0) e.pos[r] = p;
  const float* src = e.wte + (size_t)tok * e.E;
  const float* pe = e.wpe ? e.wpe + (size_t)p * e.E : nullptr;
  float* dst = e.x + (size_t)r * e.E;
  bf16* db = e.xb + (size_t)r * e.ldxb;
  for (int j = threadIdx.x; j < e.E; j += blockDim.x) {
    const float v = pe ? src[j] + pe[j] : src[j];
    dst[j] = v;
    db[j] = __float2bfloat16_rn(v);
  }
}

// ---- decode attention over the paged cache (AttendRow, CachedRowMath.ts:60-86) ---------------------
// Grid (split, kv head, row). Row m attends over positions 0..pos[m] of its slot. Each CTA streams the
// pages of its split [c * pages / nsplit, (c + 1) * pages / nsplit) through a ring of shared-memory
// buffers filled by bulk async copies (one thread issues the K and V block copies of a page), scores each
// page against the head's whole query group (GQA: heads g*G .. g*G+G-1 share it) and keeps an online
// softmax (running max and sum, rescaled output). One split writes the context directly; with several
// splits each writes a partial (o, max, sum) and the last split of a (row, kv head) to finish — counted
// with an atomic — merges them in split order.

struct AttnArgs {
  const float* q;   // [M, H*d] post-RoPE
  float* ctx;       // [M, H*d]
  bf16* ctxb;       // [M, ldcb]
  int ldcb;
  KvView kv;
  int layer;
  const int* pos;
  const int* slot;
  int H, Hk, G, d;
  float scale;
  int max_chunks;   // partial stride (>= gridDim.x)
  float* part_o;    // [M, H, max_chunks, d]
  float* part_m;    // [M, H, max_chunks]
  float* part_l;
  int* counter;     // [M, Hk], zero between launches
};

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kMaxGroup = 8;
constexpr int kAttnRing = 3;  // page buffers in flight per CTA

__device__ __forceinline__ void StoreCtx(const AttnArgs& aa, int m, int col, float v) {
  if (aa.ctx) aa.ctx[(size_t)m * aa.H * aa.d + col] = v;
  aa.ctxb[(size_t)m * aa.ldcb + col] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ void AttnMerge(const AttnArgs& aa, int m, int g, int nsplit) {
  for (int e = threadIdx.x; e < aa.G * aa.d; e += blockDim.x) {
    const int i = e / aa.d, j = e % aa.d;
    const int h = g * aa.G + i;
    const size_t base = ((size_t)m * aa.H + h) * aa.max_chunks;
    float mx = -INFINITY;
    for (int c = 0; c < nsplit; c++) mx = fmaxf(mx, __ldcg(aa.part_m + base + c));
    float num = 0.f, den = 0.f;
    for (int c = 0; c < nsplit; c++) {
      const float pm = __ldcg(aa.part_m + base + c);
      const float w = pm == -INFINITY ? 0.f : __expf(pm - mx);
      num += w * __ldcg(aa.part_o + (base + c) * aa.d + j);
      den += w * __ldcg(aa.part_l + base + c);
    }
    StoreCtx(aa, m, h * aa.d + j, num / den);
  }
}

// Writes this CTA's per-head results (so = unnormalized output [G*d], sm/sl = running max/sum); merges
// when it is the last split of its (row, kv head).
__device__ __forceinline__ void AttnFinishSplit(const AttnArgs& aa, int m, int g, const float* so, const float* sm,
                                                const float* sl) {
  const int c = blockIdx.x, nsplit = gridDim.x;
  if (nsplit == 1) {
    for (int e = threadIdx.x; e < aa.G * aa.d; e += blockDim.x) {
      const int i = e / aa.d, j = e % aa.d;
      StoreCtx(aa, m, (g * aa.G + i) * aa.d + j, so[e] / sl[i]);
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
    s_last = (prev == nsplit - 1);
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    AttnMerge(aa, m, g, nsplit);
    if (threadIdx.x == 0) aa.counter[m * aa.Hk + g] = 0;
  }
}

// One-dimensional bulk async copy global -> shared (16-byte aligned, size a multiple of 16), counted on bar.
__device__ __forceinline__ void BulkCopyG2S(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   SmemAddr(dst)),
               "l"(src), "r"(bytes), "r"(SmemAddr(bar))
               : "memory");
}

// Ampere-style 16-byte asynchronous copy global -> shared (both addresses 16-byte aligned), L2 only.
__device__ __forceinline__ void CpAsync16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(SmemAddr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void CpAsyncCommit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void CpAsyncWaitAll() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__host__ __device__ constexpr int AttnSmemBytes(int D) { return kAttnRing * 2 * kPageTokens * D * 2; }

// Fast path: head_dim D (multiple of 8, 32..128) known at compile time. Dynamic shared memory holds the
// ring of K|V page buffers.
template <int D>
__global__ void __launch_bounds__(kAttnThreads) AttnDecodeKernel(AttnArgs aa) {
  constexpr int JPL = D / 32;   // output dims per lane
  constexpr int PAGE = kPageTokens * D;  // elements of one K (or V) page
  extern __shared__ __align__(128) uint8_t attn_smem[];
  bf16* ring = reinterpret_cast<bf16*>(attn_smem);  // [kAttnRing][K page | V page]
  __shared__ __align__(8) uint64_t bar[kAttnRing];
  __shared__ __align__(16) float sq[kMaxGroup][D];
  __shared__ float ss[kMaxGroup][kPageTokens];
  __shared__ float so[kMaxGroup * D];
  __shared__ float s_m[kMaxGroup], s_l[kMaxGroup], s_scale[kMaxGroup];
  __shared__ int s_fail;
  static_assert(kAttnWarps * kMaxGroup * D * 4 <= kAttnRing * 2 * PAGE * 2, "partials must fit in the ring");
  GridDepWait();
  GridDepLaunch();
  const int g = blockIdx.y, m = blockIdx.z;
  const int p = aa.pos[m];
  const int pages = (p + kPageTokens) / kPageTokens;  // positions 0..p
  const int pb = (int)((long long)blockIdx.x * pages / gridDim.x);
  const int pe = (int)((long long)(blockIdx.x + 1) * pages / gridDim.x);
  const int G = aa.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = aa.H * D;
  const int slot = aa.slot[m];

  if (threadIdx.x == 0) {
    for (int b = 0; b < kAttnRing; b++) MbarInit(&bar[b], 1);
    FenceMbarInit();
    s_fail = 0;
  }
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) sq[e / D][e % D] = aa.q[(size_t)m * hd + g * G * D + e];
  if (threadIdx.x < kMaxGroup) {
    s_m[threadIdx.x] = -INFINITY;
    s_l[threadIdx.x] = 0.f;
  }
  __syncthreads();
  // Positions held by page `pg` (0 when its block is missing: the miss is recorded as an error).
  auto page_len = [&](int pg) { return min(kPageTokens, p + 1 - pg * kPageTokens); };
  auto issue = [&](int pg, int b) {
    const bf16* kb = aa.kv.Block(slot, pg, aa.layer, g, 0);
    const bf16* vb = aa.kv.Block(slot, pg, aa.layer, g, 1);
    if (kb == nullptr) {
      MbarArrive(&bar[b]);  // complete the phase with no data
      return;
    }
    const uint32_t bytes = (uint32_t)page_len(pg) * D * 2;
    MbarArriveExpectTx(&bar[b], 2 * bytes);
    BulkCopyG2S(ring + (size_t)b * 2 * PAGE, kb, bytes, &bar[b]);
    BulkCopyG2S(ring + (size_t)b * 2 * PAGE + PAGE, vb, bytes, &bar[b]);
  };
  if (threadIdx.x == 0) {
    FenceProxyAsyncGlobal();
    for (int pg = pb; pg < pe && pg < pb + kAttnRing; pg++) issue(pg, (pg - pb) % kAttnRing);
  }

  float o[kMaxGroup][JPL];
#pragma unroll
  for (int i = 0; i < kMaxGroup; i++)
#pragma unroll
    for (int jj = 0; jj < JPL; jj++) o[i][jj] = 0.f;
  for (int pg = pb; pg < pe; pg++) {
    const int it = pg - pb, b = it % kAttnRing;
    const bool present = aa.kv.block_table[slot * aa.kv.max_blocks + pg] >= 0;
    if (!MbarWaitBounded(&bar[b], (it / kAttnRing) & 1, kWaitLimit)) {
      atomicCAS(&g_shahd_device_error, 0, kDevErrAttnTimeout);
      s_fail = 1;
    }
    __syncthreads();
    if (s_fail) break;  // uniform: read after the barrier
    const int tv = present ? page_len(pg) : 0;
    const bf16* sk = ring + (size_t)b * 2 * PAGE;
    const bf16* sv = sk + PAGE;
    // scores s[i][t] = (q_i · k_t) * scale. Warp w scores positions 16w .. 16w + 15, two lanes per
    // position (each half of the head dimension); lane l starts its half at pair (c + l) mod D/4, so the
    // 32 lanes read 32 different banks of the K rows and one shuffle joins the halves.
    {
      constexpr int HW = D / 4;  // bf16 pairs per half row
      static_assert(kAttnWarps * 16 == kPageTokens, "one position per lane pair");
      const int t = warp * 16 + (lane & 15), h = lane >> 4;
      const __nv_bfloat162* krow = reinterpret_cast<const __nv_bfloat162*>(sk) + t * (D / 2) + h * HW;
      for (int i = 0; i < G; i++) {
        const float2* qh = reinterpret_cast<const float2*>(&sq[i][0]) + h * HW;
        float a = 0.f, b = 0.f;
#pragma unroll
        for (int c = 0; c < HW; c++) {
          const int wd = (c + lane) & (HW - 1);
          const float2 kf = __bfloat1622float2(krow[wd]);
          const float2 qv = qh[wd];
          a = fmaf(kf.x, qv.x, a);
          b = fmaf(kf.y, qv.y, b);
        }
        a += b;
        a += __shfl_xor_sync(0xffffffffu, a, 16);
        if (h == 0 && t < tv) ss[i][t] = a * aa.scale;  // rows past tv hold stale data: never stored
      }
    }
    __syncthreads();
    // online softmax update per head
    for (int i = warp; i < G; i += kAttnWarps) {
      float pm = -INFINITY;
      for (int t = lane; t < tv; t += 32) pm = fmaxf(pm, ss[i][t]);
      pm = WarpMax(pm);
      const float old = s_m[i];
      const float nm = fmaxf(old, pm);
      float sum = 0.f;
      for (int t = lane; t < tv; t += 32) {
        const float e = __expf(ss[i][t] - nm);
        ss[i][t] = e;
        sum += e;
      }
      sum = WarpSum(sum);
      if (lane == 0) {
        const float sc = old == -INFINITY ? 0.f : __expf(old - nm);
        s_scale[i] = sc;
        s_l[i] = s_l[i] * sc + sum;
        s_m[i] = nm;
      }
    }
    __syncthreads();
    // o = o * scale + sum_t e[i][t] * v_t; warps split t, lanes split j
#pragma unroll
    for (int i = 0; i < kMaxGroup; i++)
      if (i < G) {
        const float sc = s_scale[i];
#pragma unroll
        for (int jj = 0; jj < JPL; jj++) o[i][jj] *= sc;
      }
#pragma unroll 4
    for (int t = warp; t < tv; t += kAttnWarps) {
      float vf[JPL];
      if constexpr (JPL == 2) {
        const float2 v2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sv + t * D + lane * 2));
        vf[0] = v2.x;
        vf[1] = v2.y;
      } else {
#pragma unroll
        for (int jj = 0; jj < JPL; jj++) vf[jj] = __bfloat162float(sv[t * D + lane * JPL + jj]);
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
    __syncthreads();  // buffer b and ss are free again
    if (threadIdx.x == 0 && pg + kAttnRing < pe) issue(pg + kAttnRing, b);
  }
  // combine the warps' partial outputs (the ring is free now)
  float* so_part = reinterpret_cast<float*>(ring);  // [warps][kMaxGroup * D]
#pragma unroll
  for (int i = 0; i < kMaxGroup; i++)
    if (i < G)
#pragma unroll
      for (int jj = 0; jj < JPL; jj++) so_part[(warp * kMaxGroup + i) * D + lane * JPL + jj] = o[i][jj];
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) acc += so_part[w * kMaxGroup * D + e];
    so[e] = acc;
  }
  __syncthreads();
  AttnFinishSplit(aa, m, g, so, s_m, s_l);
}

// ---- decode-step attention with the cache read ahead of the predecessor --------------------------------
// In a decode step every row appends exactly one position (its own slot): the K/V rows of positions
// 0 .. p-1 were written by earlier steps, the block table and the row's position and slot by earlier
// launches. With programmatic dependent launch this kernel starts once the QKV projection of the layer has
// passed its own grid-dependency wait, i.e. after every launch before that projection has completed, so
// all of those are read before this kernel's wait, and only q and the K/V row at p (written by the
// projection) after it. The cached rows then arrive while the projection still runs.
//
// One CTA of 8 warps per (split, kv head, row); a warp task is 32 consecutive positions. A task's K and V
// rows are read as coalesced 16-byte chunks: with C = D/8 chunks per row, load i (i < C) gives lane l
// chunk l % C of row i*(32/C) + l/C, so each load instruction covers 32/C whole rows. Scores: each lane
// dots its chunks with q, and a reduce-scatter over the C lanes of a row group leaves lane l with the full
// score of row (l % C)*(32/C) + l/C. P.V: lane l accumulates its chunk's 8 dims over its rows (the
// probability of row r comes from the lane that scored it); the row groups are summed once at the end.
// Each warp keeps a running max and sum per head; the warps' states merge in shared memory, the splits
// through AttnFinishSplit.
constexpr int kAttnRowWarps = 8;  // the most warps a CTA has (shared memory is sized for them)
constexpr int kAttnTask = 32;  // positions per warp task (a task never straddles a 64-position page)

__host__ __device__ constexpr int AttnRowsSmem(int G, int D) {
  // q [G][D] (reused for the merged output), warp outputs [warps][G][D], warp max/sum, merged max/sum
  return (G * D + kAttnRowWarps * G * D + 2 * kAttnRowWarps * G + 2 * G) * 4;
}

__device__ __forceinline__ void PrefetchL2(const void* ptr) { asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr)); }

// Sum over the C lanes of a row group (lanes l ^ k, k < C) of C values per lane, scattered: lane l ends
// with the total of value index l % C. C is a power of two.
template <int C>
__device__ __forceinline__ float ReduceScatter(float (&v)[C], int lane) {
#pragma unroll
  for (int o = C / 2; o >= 1; o /= 2) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int k = 0; k < o; k++) {
      const float send = up ? v[k] : v[k + o];
      const float keep = up ? v[k + o] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

// Eight bf16 (a 16-byte chunk) to fp32 by moving each half into the high bits.
__device__ __forceinline__ void Bf16ChunkToFloat(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; k++) {
    f[2 * k] = __uint_as_float(w[k] << 16);
    f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
}

// MG: a power of two >= G (per-head state lives in registers sized by it); NW warps per CTA: 8 while
// the grid fits two CTAs per SM, 4 for many rows, so that more rows are resident at once.
template <int D, int MG, int NW>
__global__ void __launch_bounds__(NW * 32, (D <= 64 && MG <= 2 ? 2 : 1) * (8 / NW)) AttnRowsKernel(AttnArgs aa) {
  constexpr int C = D / 8;            // 16-byte chunks per row
  constexpr int RPI = kAttnTask / C;  // rows per load instruction
  extern __shared__ __align__(16) float ar_smem[];
  const int G = aa.G;
  float* sq = ar_smem;                     // [G][D] q pre-scaled; later the merged output
  float* wo = sq + G * D;                  // [warps][G][D]
  float* wm = wo + NW * G * D;  // [warps][G]
  float* wl = wm + NW * G;      // [warps][G]
  float* mm = wl + NW * G;      // [G]
  float* ml = mm + G;                      // [G]
  const int g = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ck = lane % C, rg = lane / C;  // this lane's chunk and row group

  // ---- before the wait: launches older than the predecessor only ----
  const int p = __ldcg(aa.pos + m), slot = __ldcg(aa.slot + m);
  const int ntask = p / kAttnTask + 1;
  const int per = CeilDiv(ntask, (int)gridDim.x);
  const int c0 = blockIdx.x * per, c1 = min(ntask, c0 + per);
  const size_t head_off = (size_t)((aa.layer * aa.Hk + g) * 2) * kPageTokens * D;
  // K rows of task c (position c*32 + row; its V rows follow one K page later); nullptr when the page is
  // missing (recorded as an error)
  auto task_base = [&](int c) -> const bf16* {
    const int page = __ldcg(aa.kv.block_table + (size_t)slot * aa.kv.max_blocks + (c * kAttnTask) / kPageTokens);
    if (page < 0) {
      atomicCAS(&g_shahd_device_error, 0, kDevErrNoPage);
      return nullptr;
    }
    return aa.kv.pool + (size_t)page * aa.kv.page_elems + head_off + (size_t)((c * kAttnTask) % kPageTokens) * D;
  };
  uint4 kr[C], vr[C];  // chunk ck of rows i*RPI + rg
#pragma unroll
  for (int i = 0; i < C; i++) kr[i] = vr[i] = make_uint4(0, 0, 0, 0);
  // rows of task c at positions [lo, hi)
  auto load_rows = [&](const bf16* kb, int c, int lo, int hi) {
    const int t0 = c * kAttnTask;
    const uint4* kp = reinterpret_cast<const uint4*>(kb) + ck;
    const uint4* vp = reinterpret_cast<const uint4*>(kb + (size_t)kPageTokens * D) + ck;
#pragma unroll
    for (int i = 0; i < C; i++) {
      const int r = i * RPI + rg;
      if (t0 + r >= lo && t0 + r < hi) {
        kr[i] = __ldcg(kp + (size_t)r * C);
        vr[i] = __ldcg(vp + (size_t)r * C);
      }
    }
  };
  int c = c0 + warp;
  const bf16* kb = c < c1 ? task_base(c) : nullptr;
  if (kb) load_rows(kb, c, 0, p);
  for (int cc = c + NW; cc < c1; cc += NW) {  // later tasks of this warp: into L2
    const bf16* b = task_base(cc);
    if (b) {
      for (int i = lane; i < kAttnTask * D * 2 / 128; i += 32) {  // one 128-byte line per lane and load
        PrefetchL2(reinterpret_cast<const char*>(b) + (size_t)i * 128);
        PrefetchL2(reinterpret_cast<const char*>(b + (size_t)kPageTokens * D) + (size_t)i * 128);
      }
    }
  }

  GridDepWait();
  GridDepLaunch();
  // ---- after the wait: q and the row at p ----
  const int hd = aa.H * D;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) sq[e] = __ldcg(aa.q + (size_t)m * hd + g * G * D + e) * aa.scale;
  if (kb) load_rows(kb, c, p, p + 1);
  __syncthreads();

  float o[MG][8], mrun[MG], lrun[MG];
#pragma unroll
  for (int h = 0; h < MG; h++) {
    mrun[h] = -INFINITY;
    lrun[h] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) o[h][j] = 0.f;
  }
  for (bool first = true; c < c1; c += NW, first = false) {
    const int t0 = c * kAttnTask;
    if (!first) {
      kb = task_base(c);
#pragma unroll
      for (int i = 0; i < C; i++) kr[i] = vr[i] = make_uint4(0, 0, 0, 0);  // rows past p stay zero
      if (kb) load_rows(kb, c, 0, p + 1);
    }
    if (kb == nullptr) continue;  // missing page: its positions are left out (the error flag is set)
    const bool valid = t0 + ck * RPI + rg <= p;  // the row this lane scores
    float pv[MG];
#pragma unroll
    for (int h = 0; h < MG; h++) {
      pv[h] = 0.f;
      if (h < G) {
        const float4 q0 = *reinterpret_cast<const float4*>(sq + h * D + ck * 8);
        const float4 q1 = *reinterpret_cast<const float4*>(sq + h * D + ck * 8 + 4);
        const float qf[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};  // this lane's q chunk
        float part[C];
#pragma unroll
        for (int i = 0; i < C; i++) {
          float kf[8];
          Bf16ChunkToFloat(kr[i], kf);
          float a = 0.f;
#pragma unroll
          for (int j = 0; j < 8; j++) a = fmaf(qf[j], kf[j], a);
          part[i] = a;
        }
        const float full = ReduceScatter<C>(part, lane);  // every lane takes part in the shuffles
        const float si = valid ? full : -INFINITY;
        // online softmax (position c*32 <= p, so every task has a finite max)
        const float nm = fmaxf(mrun[h], WarpMax(si));
        const float sc = mrun[h] == -INFINITY ? 0.f : __expf(mrun[h] - nm);
        pv[h] = valid ? __expf(si - nm) : 0.f;
        lrun[h] = lrun[h] * sc + pv[h];
#pragma unroll
        for (int j = 0; j < 8; j++) o[h][j] *= sc;
        mrun[h] = nm;
      }
    }
    // o += p_r v_r over this lane's rows r = i*RPI + rg, scored by lane rg*C + i (rows past p are zero)
#pragma unroll
    for (int i = 0; i < C; i++) {
      float vf[8];
      Bf16ChunkToFloat(vr[i], vf);
#pragma unroll
      for (int h = 0; h < MG; h++) {
        if (h < G) {
          const float pt = __shfl_sync(0xffffffffu, pv[h], rg * C + i);
#pragma unroll
          for (int j = 0; j < 8; j++) o[h][j] = fmaf(pt, vf[j], o[h][j]);
        }
      }
    }
  }
  // the warps' states (row groups summed), then their merge (weights exp(m_w - M); idle warps: m_w = -inf)
#pragma unroll
  for (int h = 0; h < MG; h++) {
    if (h < G) {
#pragma unroll
      for (int j = 0; j < 8; j++)
#pragma unroll
        for (int off = C; off < 32; off *= 2) o[h][j] += __shfl_xor_sync(0xffffffffu, o[h][j], off);
      const float l = WarpSum(lrun[h]);
      if (lane == 0) {
        wm[warp * G + h] = mrun[h];
        wl[warp * G + h] = l;
      }
      if (rg == 0) {
#pragma unroll
        for (int j = 0; j < 8; j++) wo[(warp * G + h) * D + ck * 8 + j] = o[h][j];
      }
    }
  }
  __syncthreads();
  if (gridDim.x == 1) {  // one split: every thread merges the warps for its outputs and stores them
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
      const int i = e / D;
      float M = -INFINITY, L = 0.f, acc = 0.f;
      for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w * G + i]);
      for (int w = 0; w < NW; w++)
        if (wm[w * G + i] != -INFINITY) L += __expf(wm[w * G + i] - M) * wl[w * G + i];
      for (int w = 0; w < NW; w++)
        if (wm[w * G + i] != -INFINITY) acc += __expf(wm[w * G + i] - M) * wo[(w * G + i) * D + e % D];
      StoreCtx(aa, m, (g * G + i) * D + e % D, acc / L);
    }
    return;
  }
  if (threadIdx.x < G) {
    const int i = threadIdx.x;
    float M = -INFINITY, L = 0.f;
    for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w * G + i]);
    for (int w = 0; w < NW; w++)
      if (wm[w * G + i] != -INFINITY) L += __expf(wm[w * G + i] - M) * wl[w * G + i];
    mm[i] = M;
    ml[i] = L;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int i = e / D;
    float acc = 0.f;
    for (int w = 0; w < NW; w++)
      if (wm[w * G + i] != -INFINITY) acc += __expf(wm[w * G + i] - mm[i]) * wo[(w * G + i) * D + e % D];
    sq[e] = acc;
  }
  __syncthreads();
  AttnFinishSplit(aa, m, g, sq, mm, ml);
}

// Any even head_dim up to 128 (the reference's small test shapes use d = 4, 8, 16): scalar loops over
// global memory, one split per (row, kv head), online softmax over the pages.
constexpr int kMaxHeadDimGeneric = 128;
__global__ void __launch_bounds__(kAttnThreads) AttnDecodeGenericKernel(AttnArgs aa) {
  __shared__ float sq[kMaxGroup * kMaxHeadDimGeneric];
  __shared__ float ss[kMaxGroup][kPageTokens];
  __shared__ float so[kMaxGroup * kMaxHeadDimGeneric];
  __shared__ float s_m[kMaxGroup], s_l[kMaxGroup], s_scale[kMaxGroup];
  GridDepWait();
  GridDepLaunch();
  const int g = blockIdx.y, m = blockIdx.z;
  const int p = aa.pos[m];
  const int pages = (p + kPageTokens) / kPageTokens;
  const int pb = (int)((long long)blockIdx.x * pages / gridDim.x);
  const int pe = (int)((long long)(blockIdx.x + 1) * pages / gridDim.x);
  const int G = aa.G, D = aa.d;
  const int hd = aa.H * D;
  const int slot = aa.slot[m];
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    sq[e] = aa.q[(size_t)m * hd + g * G * D + e];
    so[e] = 0.f;
  }
  if (threadIdx.x < kMaxGroup) {
    s_m[threadIdx.x] = -INFINITY;
    s_l[threadIdx.x] = 0.f;
  }
  __syncthreads();
  for (int pg = pb; pg < pe; pg++) {
    const bf16* kb = aa.kv.Block(slot, pg, aa.layer, g, 0);
    const bf16* vb = aa.kv.Block(slot, pg, aa.layer, g, 1);
    const int tv = kb ? min(kPageTokens, p + 1 - pg * kPageTokens) : 0;
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
      float pm = -INFINITY;
      for (int t = 0; t < tv; t++) pm = fmaxf(pm, ss[i][t]);
      const float old = s_m[i], nm = fmaxf(old, pm);
      float sum = 0.f;
      for (int t = 0; t < tv; t++) {
        const float e = __expf(ss[i][t] - nm);
        ss[i][t] = e;
        sum += e;
      }
      const float sc = old == -INFINITY ? 0.f : __expf(old - nm);
      s_scale[i] = sc;
      s_l[i] = s_l[i] * sc + sum;
      s_m[i] = nm;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
      const int i = e / D, j = e % D;
      float acc = so[e] * s_scale[i];
      for (int t = 0; t < tv; t++) acc = fmaf(ss[i][t], __bfloat162float(vb[(size_t)t * D + j]), acc);
      so[e] = acc;
    }
    __syncthreads();
  }
  AttnFinishSplit(aa, m, g, so, s_m, s_l);
}

// ---- finish: positions advance; greedy argmax over the head's per-CTA partials -------------------------

struct FinishArgs {
  int M;
  const int* slot;
  int* pos;
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
  // decode loop only (wte != nullptr): embed each row's chosen id as the next step's input and advance its
  // position, so that step needs no embed kernel (rows whose window is full are left to the rebuild)
  const float* wte;
  const float* wpe;  // nullptr for RoPE models
  float* x;
  bf16* xb;
  int E, ldxb, C;
};

__global__ void FinishKernel(FinishArgs f) {
  GridDepWait();
  GridDepLaunch();
  const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= f.M) return;
  if (lane == 0) f.seq_len[f.slot[r]] = f.pos[r] + 1;
  if (f.am_val == nullptr && f.sampled == nullptr) return;
  int id;
  if (f.sampled) {
    id = f.sampled[r];
  } else {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int b = lane; b < f.nblk; b += 32) ArgmaxMerge(bv, bi, f.am_val[(size_t)r * f.nblk + b], f.am_idx[(size_t)r * f.nblk + b]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      ArgmaxMerge(bv, bi, ov, oi);
    }
    id = bi == 0x7fffffff ? 0 : bi;
  }
  if (f.wte != nullptr) {  // EmbeddingLookup (+ learned position) of the next step's token, Embedding.ts:14-26
    const int np = f.pos[r] + 1;
    if (np < f.C) {
      const float* src = f.wte + (size_t)id * f.E;
      const float* pe = f.wpe ? f.wpe + (size_t)np * f.E : nullptr;
      for (int j = lane; j < f.E; j += 32) {
        const float v = pe ? src[j] + pe[j] : src[j];
        f.x[(size_t)r * f.E + j] = v;
        f.xb[(size_t)r * f.ldxb + j] = __float2bfloat16_rn(v);
      }
    }
    __syncwarp();
    if (lane == 0) f.pos[r] = np;
  }
  if (lane != 0) return;
  if (f.next_ids) f.next_ids[r] = id;
  if (f.cur_tok) f.cur_tok[r] = id;
  if (f.out_ids) {
    const int k = f.gen_count[r];
    f.out_ids[(size_t)r * f.out_ld + k] = id;
    f.gen_count[r] = k + 1;
  }
}

}  // namespace shahd
