// FusedAttention as an operator on given Q, K, V: the attention core of MultiHeadAttention.Forward
// (Brain/Nn/MultiHeadAttention.ts:46-74: ApplyRope on Q and K, MatMulNT(Q, K), CausalSoftmax(., scale),
// MatMul(., V), GQA head h reading kv head h / (H / Hk)) for a batched causal prefill, then 1-token decode
// steps (AttendRow, Brain/Sampling/CachedRowMath.ts:60-86) over the cached rows. The K rows (after RoPE)
// and V rows live in a device-resident paged cache of the decode session's layout (one layer); the
// attention runs on the session's kernels: the tensor-core prefill kernel (head_dim 64, CUDA-core tile
// kernel otherwise) and the decode-row kernels with the session's automatic choice.
#pragma once

#include "attn_pages.cuh"
#include "decode_kernels.cuh"
#include "prefill_attention.cuh"
#include "prefill_attention_umma.cuh"

namespace shahd {

struct AttentionOp {
  std::mutex mu;
  int device = 0, max_seqs = 0, H = 0, Hk = 0, G = 0, d = 0, C = 0, max_blocks = 0, num_sms = 0;
  float scale = 0.f;
  bool rope = false;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  bf16* pool = nullptr;  // [max_seqs * max_blocks pages][Hk][K|V][64][d]; slot s owns pages s*max_blocks ..
  size_t page_elems = 0;
  int* d_block_table = nullptr;
  int* d_len = nullptr;  // cached positions per slot
  int* d_slot = nullptr;  // identity 0 .. max_seqs-1 (decode rows are slots 0..n-1)
  int* d_plan = nullptr;  // prefill plan [5][max_seqs]
  int* h_plan = nullptr;  // pinned
  std::vector<int> h_len;
  float *rope_cos = nullptr, *rope_sin = nullptr;  // [C, d/2]
  float* q_rot = nullptr;  // [rows, H*d] queries after RoPE
  bf16* ctxb = nullptr;    // [rows, H*d] bf16 copy the attention kernels also write
  size_t rows_cap = 0;
  float *part_o = nullptr, *part_m = nullptr, *part_l = nullptr;
  int* counter = nullptr;
  CUtensorMap kv_tmap;
  bool kv_tmap_ok = false;
  KvView kv() const { return KvView{pool, d_block_table, max_blocks, Hk, d, page_elems}; }
};

// RoPE (RotaryEmbedding.ts:63-75: pairs (2i, 2i+1) rotated by position * base^(-2i/d)) on the query and key
// rows of row r = (sequence s, position base[s] + r % T); queries to q_rot (fp32), keys (after RoPE) and
// values to the sequence's cache page (bf16).
__global__ void AttnRopeAppendKernel(const float* q, const float* k, const float* v, int T, const int* base,
                                     const float* rope_cos, const float* rope_sin, int H, int Hk, int d, KvView kv,
                                     float* q_rot) {
  const int r = blockIdx.x, s = r / T;
  const int pos = (base ? base[s] : 0) + r % T;
  const int half = d / 2;
  for (int e = threadIdx.x; e < (H + Hk) * half; e += blockDim.x) {
    const int h = e / half, i = e % half;
    const float* src = h < H ? q + ((size_t)r * H + h) * d : k + ((size_t)r * Hk + (h - H)) * d;
    float x0 = src[2 * i], x1 = src[2 * i + 1];
    if (rope_cos) {
      const float c = rope_cos[(size_t)pos * half + i], sn = rope_sin[(size_t)pos * half + i];
      const float y0 = x0 * c - x1 * sn, y1 = x0 * sn + x1 * c;
      x0 = y0;
      x1 = y1;
    }
    if (h < H) {
      q_rot[((size_t)r * H + h) * d + 2 * i] = x0;
      q_rot[((size_t)r * H + h) * d + 2 * i + 1] = x1;
    } else {
      const long long o = kv.Offset(s, pos, 0, h - H, 0);
      if (o >= 0) *reinterpret_cast<__nv_bfloat162*>(kv.pool + o + 2 * i) = __floats2bfloat162_rn(x0, x1);
    }
  }
  for (int e = threadIdx.x; e < Hk * d; e += blockDim.x) {
    const int g = e / d, j = e % d;
    const long long o = kv.Offset(s, pos, 0, g, 1);
    if (o >= 0) kv.pool[o + j] = __float2bfloat16_rn(v[((size_t)r * Hk + g) * d + j]);
  }
}

__global__ void AttnSetLengthKernel(int* len, int n, int value) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) len[i] = value;
}

__global__ void AttnAdvanceKernel(int* len, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) len[i] += 1;
}

template <class T>
int OpAlloc(AttentionOp* a, T** p, size_t count) {
  void* v = nullptr;
  const cudaError_t e = cudaMalloc(&v, std::max<size_t>(1, count) * sizeof(T));
  if (e != cudaSuccess) {
    SetError("cudaMalloc of %zu bytes failed: %s", count * sizeof(T), cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? SHAHD_ENOMEM : SHAHD_ECUDA;
  }
  a->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return SHAHD_OK;
}

void OpFree(AttentionOp* a) {
  cudaSetDevice(a->device);
  if (a->stream) cudaStreamSynchronize(a->stream);
  for (void* p : a->allocs) {
    if (p == a->pool) ForgetTmaRange(a->pool, reinterpret_cast<char*>(a->pool) + a->page_elems * 2 * a->max_seqs * a->max_blocks);
    cudaFree(p);
  }
  a->allocs.clear();
  if (a->h_plan) cudaFreeHost(a->h_plan);
  if (a->stream) cudaStreamDestroy(a->stream);
}

int OpGrowRows(AttentionOp* a, size_t rows) {
  if (rows <= a->rows_cap) return SHAHD_OK;
  for (void* p : {static_cast<void*>(a->q_rot), static_cast<void*>(a->ctxb)}) {
    if (!p) continue;
    cudaFree(p);
    a->allocs.erase(std::find(a->allocs.begin(), a->allocs.end(), p));
  }
  a->q_rot = nullptr;
  a->ctxb = nullptr;
  a->rows_cap = 0;
  SHAHD_TRY(OpAlloc(a, &a->q_rot, rows * a->H * a->d));
  SHAHD_TRY(OpAlloc(a, &a->ctxb, rows * a->H * a->d));
  a->rows_cap = rows;
  return SHAHD_OK;
}

}  // namespace shahd

struct ShahdAttention : shahd::AttentionOp {};

extern "C" {

int shahd_attention_create(int32_t max_seqs, int32_t num_heads, int32_t kv_heads, int32_t head_dim, int32_t capacity,
                           double rope_base, int32_t device, ShahdAttention** out) {
  using namespace shahd;
  if (!out) {
    SetError("shahd_attention_create: out is null");
    return SHAHD_EINVAL;
  }
  *out = nullptr;
  if (max_seqs < 1 || num_heads < 1 || kv_heads < 1 || num_heads % kv_heads != 0 || num_heads / kv_heads > kMaxGroup ||
      !(head_dim == 32 || head_dim == 64 || head_dim == 128) || capacity < 1) {
    SetError("shahd_attention_create: need max_seqs >= 1, kv_heads dividing num_heads with at most %d query heads "
             "per kv head, head_dim 32, 64 or 128, capacity >= 1", kMaxGroup);
    return SHAHD_EINVAL;
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    SetError("shahd_attention_create: no CUDA device %d", device);
    return SHAHD_EINVAL;
  }
  SHAHD_CUDA_TRY(cudaSetDevice(device));
  ShahdAttention* a = new ShahdAttention();
  auto fail = [&](int rc) {
    OpFree(a);
    delete a;
    return rc;
  };
  a->device = device;
  a->max_seqs = max_seqs;
  a->H = num_heads;
  a->Hk = kv_heads;
  a->G = num_heads / kv_heads;
  a->d = head_dim;
  a->C = capacity;
  a->max_blocks = CeilDiv(capacity, kPageTokens);
  a->scale = (float)(1.0 / std::sqrt((double)head_dim));
  a->rope = rope_base > 0;
  cudaDeviceGetAttribute(&a->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (cudaStreamCreateWithFlags(&a->stream, cudaStreamNonBlocking) != cudaSuccess) {
    SetError("shahd_attention_create: cudaStreamCreate failed");
    return fail(SHAHD_ECUDA);
  }
  a->page_elems = (size_t)kv_heads * 2 * kPageTokens * head_dim;
  const size_t pages = (size_t)max_seqs * a->max_blocks;
  int rc;
  if ((rc = OpAlloc(a, &a->pool, a->page_elems * pages)) != SHAHD_OK) return fail(rc);
  cudaMemset(a->pool, 0, a->page_elems * pages * sizeof(bf16));
  std::vector<int> table(pages), ids(max_seqs);
  std::iota(table.begin(), table.end(), 0);  // slot s owns pages s*max_blocks .. s*max_blocks + max_blocks-1
  std::iota(ids.begin(), ids.end(), 0);
  if ((rc = OpAlloc(a, &a->d_block_table, pages)) != SHAHD_OK || (rc = OpAlloc(a, &a->d_len, max_seqs)) != SHAHD_OK ||
      (rc = OpAlloc(a, &a->d_slot, max_seqs)) != SHAHD_OK || (rc = OpAlloc(a, &a->d_plan, 5 * (size_t)max_seqs)) != SHAHD_OK ||
      (rc = OpAlloc(a, &a->part_o, (size_t)max_seqs * num_heads * a->max_blocks * head_dim)) != SHAHD_OK ||
      (rc = OpAlloc(a, &a->part_m, (size_t)max_seqs * num_heads * a->max_blocks)) != SHAHD_OK ||
      (rc = OpAlloc(a, &a->part_l, (size_t)max_seqs * num_heads * a->max_blocks)) != SHAHD_OK ||
      (rc = OpAlloc(a, &a->counter, (size_t)max_seqs * kv_heads)) != SHAHD_OK)
    return fail(rc);
  if (cudaMallocHost(&a->h_plan, sizeof(int) * 5 * (size_t)max_seqs) != cudaSuccess) {
    SetError("shahd_attention_create: cudaMallocHost failed");
    return fail(SHAHD_ENOMEM);
  }
  cudaMemcpy(a->d_block_table, table.data(), sizeof(int) * pages, cudaMemcpyHostToDevice);
  cudaMemcpy(a->d_slot, ids.data(), sizeof(int) * max_seqs, cudaMemcpyHostToDevice);
  cudaMemset(a->d_len, 0, sizeof(int) * max_seqs);
  cudaMemset(a->counter, 0, sizeof(int) * (size_t)max_seqs * kv_heads);
  a->h_len.assign(max_seqs, 0);
  if (a->rope) {  // RopeFrequencies / RopeCosSin (RotaryEmbedding.ts:17-38) in f64, stored fp32 [C, d/2]
    const int half = head_dim / 2;
    std::vector<float> cs((size_t)capacity * half), sn((size_t)capacity * half);
    for (int i = 0; i < half; i++) {
      const double freq = std::pow(rope_base, (-2.0 * i) / head_dim);
      for (int pos = 0; pos < capacity; pos++) {
        cs[(size_t)pos * half + i] = (float)std::cos(pos * freq);
        sn[(size_t)pos * half + i] = (float)std::sin(pos * freq);
      }
    }
    if ((rc = OpAlloc(a, &a->rope_cos, cs.size())) != SHAHD_OK || (rc = OpAlloc(a, &a->rope_sin, sn.size())) != SHAHD_OK)
      return fail(rc);
    cudaMemcpy(a->rope_cos, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice);
    cudaMemcpy(a->rope_sin, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice);
  }
  if (head_dim == kFaD) {
    const long long rows = (long long)pages * kv_heads * 2 * kPageTokens;
    a->kv_tmap_ok = rows < (1LL << 31) && MakeTmaBf16(a->pool, (int)rows, head_dim, head_dim, kPageTokens, &a->kv_tmap);
  }
  TakeLaunchError(nullptr);
  if (!EnsureKernelAttrs((const void*)PrefillAttnUmmaKernel, kFaSmemLaunch) ||
      !EnsureKernelAttrs((const void*)PrefillAttnKernel<32>, PrefillAttnSmem(32)) ||
      !EnsureKernelAttrs((const void*)PrefillAttnKernel<64>, PrefillAttnSmem(64)) ||
      !EnsureKernelAttrs((const void*)PrefillAttnKernel<128>, PrefillAttnSmem(128)) || !EnsureAttnPagesAttrs<32>() ||
      !EnsureAttnPagesAttrs<64>() || !EnsureAttnPagesAttrs<128>()) {
    TakeLaunchError(nullptr);
    SetError("shahd_attention_create: kernel attributes could not be set on device %d", device);
    return fail(SHAHD_ECUDA);
  }
  if (cudaDeviceSynchronize() != cudaSuccess) {
    SetError("shahd_attention_create: device error during setup");
    return fail(SHAHD_ECUDA);
  }
  *out = a;
  return SHAHD_OK;
}

int shahd_attention_destroy(ShahdAttention* a) {
  if (!a) return SHAHD_OK;
  shahd::OpFree(a);
  delete a;
  return SHAHD_OK;
}

int32_t shahd_attention_length(ShahdAttention* a, int32_t slot) {
  if (!a || slot < 0 || slot >= a->max_seqs) return -1;
  std::lock_guard<std::mutex> g(a->mu);
  return a->h_len[slot];
}

// Causal prefill of n sequences of T positions (slots 0..n-1, their caches restarted at position 0).
int shahd_attention_prefill(ShahdAttention* a, const float* q, const float* k, const float* v, int32_t n, int32_t T,
                            float* out, void* stream) {
  using namespace shahd;
  if (!a || !q || !k || !v || !out) {
    SetError("shahd_attention_prefill: null argument");
    return SHAHD_EINVAL;
  }
  if (n < 1 || n > a->max_seqs || T < 1 || T > a->C) {
    SetError("shahd_attention_prefill: need 1 <= n <= %d sequences and 1 <= T <= %d positions (got n=%d, T=%d)",
             a->max_seqs, a->C, n, T);
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(a->mu);
  SHAHD_CUDA_TRY(cudaSetDevice(a->device));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : a->stream;
  SHAHD_CUDA_TRY(cudaStreamSynchronize(st));  // the pinned plan is rewritten below
  SHAHD_TRY(OpGrowRows(a, (size_t)n * T));
  const int R = a->max_seqs;
  for (int i = 0; i < n; i++) {  // slot, token start, length, row offset, base position
    a->h_plan[i] = i;
    a->h_plan[R + i] = i * T;
    a->h_plan[2 * R + i] = T;
    a->h_plan[3 * R + i] = i * T;
    a->h_plan[4 * R + i] = 0;
  }
  SHAHD_CUDA_TRY(cudaMemcpyAsync(a->d_plan, a->h_plan, sizeof(int) * 5 * R, cudaMemcpyHostToDevice, st));
  const KvView kv = a->kv();
  AttnRopeAppendKernel<<<n * T, 128, 0, st>>>(q, k, v, T, nullptr, a->rope_cos, a->rope_sin, a->H, a->Hk, a->d, kv,
                                               a->q_rot);
  const PrefillAttnArgs pa{a->q_rot, out, a->ctxb, a->H * a->d, kv, 0, a->H, a->Hk, a->G, a->scale, a->d_plan, R, 0};
  if (a->d == kFaD && g_umma_prefill_attn && a->kv_tmap_ok) {
    const FaArgs fa{a->kv_tmap, pa, 1, CeilDiv(T, kFaQ)};
    LaunchPdl(PrefillAttnUmmaKernel, dim3(fa.qblocks, a->H, n), dim3(kFaThreads), kFaSmemLaunch, st, fa);
  } else if (a->G <= kPfMaxG) {
    const dim3 pg(CeilDiv(T, kPfQ), a->Hk, n);
    if (a->d == 64) LaunchPdl(PrefillAttnKernel<64>, pg, dim3(kPfThreads), PrefillAttnSmem(64), st, pa);
    else if (a->d == 32) LaunchPdl(PrefillAttnKernel<32>, pg, dim3(kPfThreads), PrefillAttnSmem(32), st, pa);
    else LaunchPdl(PrefillAttnKernel<128>, pg, dim3(kPfThreads), PrefillAttnSmem(128), st, pa);
  } else {
    SetError("shahd_attention_prefill: more than %d query heads per kv head need head_dim 64", kPfMaxG);
    return SHAHD_EINVAL;
  }
  AttnSetLengthKernel<<<CeilDiv(n, 128), 128, 0, st>>>(a->d_len, n, T);
  for (int i = 0; i < n; i++) a->h_len[i] = T;
  return CheckLaunch("shahd_attention_prefill");
}

// One decode step for sequences 0..n-1 at their cached lengths.
int shahd_attention_decode(ShahdAttention* a, const float* q, const float* k, const float* v, int32_t n, float* out,
                           void* stream) {
  using namespace shahd;
  if (!a || !q || !k || !v || !out) {
    SetError("shahd_attention_decode: null argument");
    return SHAHD_EINVAL;
  }
  if (n < 1 || n > a->max_seqs) {
    SetError("shahd_attention_decode: need 1 <= n <= %d sequences (got %d)", a->max_seqs, n);
    return SHAHD_EINVAL;
  }
  std::lock_guard<std::mutex> g(a->mu);
  long long attended = 0;
  for (int i = 0; i < n; i++) {
    if (a->h_len[i] >= a->C) {
      SetError("shahd_attention_decode: sequence %d has filled its %d-position capacity", i, a->C);
      return SHAHD_EINVAL;
    }
    attended += a->h_len[i] + 1;
  }
  SHAHD_CUDA_TRY(cudaSetDevice(a->device));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : a->stream;
  SHAHD_TRY(OpGrowRows(a, (size_t)n));
  const KvView kv = a->kv();
  AttnRopeAppendKernel<<<n, 128, 0, st>>>(q, k, v, 1, a->d_len, a->rope_cos, a->rope_sin, a->H, a->Hk, a->d, kv,
                                           a->q_rot);
  const AttnArgs aa{a->q_rot, out, a->ctxb, a->H * a->d, kv, 0, a->d_len, a->d_slot, a->H, a->Hk, a->G, a->d,
                    a->scale, a->max_blocks, a->part_o, a->part_m, a->part_l, a->counter};
  // the decode session's choice: long rows over a grid that fills the SMs stream pages, others read ahead
  const bool long_rows = attended >= (long long)kApMinMeanLen * n && n * a->Hk >= a->num_sms;
  const bool pages = g_decode_attn_kernel == 3 || (g_decode_attn_kernel == 0 && long_rows);
  if (pages) {
    int nsplit = 1;
    if (n * a->Hk < a->num_sms) nsplit = std::max(1, std::min(a->max_blocks, CeilDiv(3 * a->num_sms, n * a->Hk)));
    LaunchAttnPages(a->d, a->G, dim3(nsplit, a->Hk, n), st, aa);
  } else {
    int rsplit = 1;
    if (n * a->Hk < a->num_sms) rsplit = std::max(1, std::min(a->max_blocks, CeilDiv(2 * a->num_sms, n * a->Hk)));
    LaunchAttnRows(a->d, a->G, dim3(rsplit, a->Hk, n), a->num_sms, st, aa);
  }
  AttnAdvanceKernel<<<CeilDiv(n, 128), 128, 0, st>>>(a->d_len, n);
  for (int i = 0; i < n; i++) a->h_len[i] += 1;
  return CheckLaunch("shahd_attention_decode");
}

}  // extern "C"
