// Fused decode attention block: one launch per layer runs the attention half of AdvanceOneToken
// (CachedForward.ts:66-84) for a batch of decode rows:
//   norm1 (NormRow, CachedRowMath.ts:25-56) -> Q/K/V projection (MatMulRow, :14-23) -> RoPE
//   (RotaryEmbedding.ts:42-60) -> K/V appended to the paged cache (KvCache.ts:60-80) -> attention over
//   positions 0..p (AttendRow, CachedRowMath.ts:60-86) -> summed per-head output projection + residual
//   (CachedForward.ts:75-84).
//
// The per-kernel chain spends three dependent launches on this (QKV projection, attention, O projection);
// at decode sizes each launch is bound by its latency (grid-dependency wait, first tile, epilogue), not by
// its bytes. Here one CTA per (kv head, row) does all of it, and the kv heads of a row form a cluster:
//   * before the grid-dependency wait: TMA loads of its kv head's Q/K/V weight rows ((G + 2) d rows, gamma
//     folded) as 128-byte swizzled boxes, and (layers after the first) the row's cached K/V rows into
//     registers / L2, exactly as AttnRowsKernel does;
//   * after the wait: the row's fp32 residual and its norm statistics (every warp, from registers), the
//     (G + 2) d projections on the tensor cores (mma m16n8k16: weight tiles by ldmatrix from the swizzled
//     boxes, the bf16 row as column 0 of B), the norm applied per output, RoPE, the new K/V row to the cache;
//   * the Wo columns of its head group ([E, G d]) are copied into the freed weight buffer (16-byte
//     asynchronous copies) while the attention runs; the context stays in shared memory (fp32) and feeds
//     this group's share of the output projection;
//   * the cluster's first CTA adds the kv heads' shares (read from the peers' shared memory) to the
//     residual in kv-head order, so the result does not depend on timing, and refreshes the bf16 copy.
// Used for decode rows when the weights of one kv head fit next to a second resident CTA (MicroChat-size
// layers) and the rows x kv heads already fill the SMs (no position splits). Every wait is bounded.
#pragma once

#include "umma_linear.cuh"

namespace shahd {

struct AttnBlockArgs {
  float* x;           // [rows, E] residual: norm input, updated by each row's cluster
  bf16* xb;           // [rows, ldxb] bf16 copy of x (the next projection's tensor-core operand)
  int E, ldxb;
  int Ep;             // padded row length of w_qkv
  const float* c1;    // LayerNorm folding per QKV column (sum_k W', beta . W); unused for RMSNorm
  const float* c2;
  int norm;           // kNormRms or kNormLayer
  float eps;
  const bf16* w_o;    // [E, HDp]: per-head Wo concatenated along the input
  int HDp;
  const float* rope_cos;  // [C, d/2] or nullptr (learned positions)
  const float* rope_sin;
  KvView kv;
  int layer;
  const int* pos;
  const int* slot;
  int H, Hk, G;
  float scale;        // 1 / sqrt(d)
  int early;          // positions, slots and cached K/V rows may be read before the grid-dependency wait
};

constexpr int kAbWarps = 8;
constexpr int kAbThreads = kAbWarps * 32;
constexpr int kAbMaxE = 512;  // residual width the warps hold in registers (two 8-float chunks per lane)

// Q/K/V weight rows of one kv head in shared memory: (G + 2) row groups of d rows (q heads, k, v), each as
// ceil(Ep / 64) TMA boxes of d rows x 64 columns in the 128-byte swizzled layout (1024-byte aligned).
__host__ __device__ constexpr int AbKBlocks(int Ep) { return (Ep + 63) / 64; }
__host__ __device__ constexpr int AbWeightBytes(int G, int D, int Ep) { return (G + 2) * AbKBlocks(Ep) * D * 128; }
__host__ __device__ constexpr int AbSmemBytes(int G, int D, int Ep) {
  return 1024 /*alignment*/ + AbWeightBytes(G, D, Ep) + 64 /*barrier*/ + AbKBlocks(Ep) * 64 * 2 /*x bf16*/ +
         (G + 2) * D * 4 /*raw projections*/ + G * D * 4 /*q*/ + 2 * D * 2 /*new k, v*/ +
         kAbWarps * G * D * 4 /*warp outputs*/ + 2 * kAbWarps * G * 4 /*warp max, sum*/ + G * D * 4 /*context*/ +
         D * 4 /*RoPE cos, sin*/ + kAbMaxE * 4 /*output-projection share*/;
}

__device__ __forceinline__ void LdMatrixX4(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}
// D[16x8] += A[16x16] (bf16, row) . B[16x8] (bf16, col), fp32 accumulators
__device__ __forceinline__ void MmaBf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
               "{%0, %1, %2, %3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t ClusterCtaRank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

template <int D, int MG>
__global__ void __launch_bounds__(kAbThreads, 2)
    AttnBlockKernel(AttnBlockArgs ab, const __grid_constant__ CUtensorMap tmap_qkv) {
  constexpr int NW = kAbWarps;
  constexpr int C = D / 8;            // 16-byte chunks per K/V row
  constexpr int RPI = kAttnTask / C;  // rows per load instruction
  extern __shared__ uint8_t ab_raw[];
  uint8_t* ab_smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ab_raw) + 1023) & ~uintptr_t(1023));
  const int G = ab.G, GD = G * D, E = ab.E, Ep = ab.Ep;
  const int nout = (G + 2) * D, nkb = AbKBlocks(Ep);
  uint8_t* sw = ab_smem;  // QKV boxes; after the projection, the Wo columns [E][G d] (plain rows)
  uint64_t* bar = reinterpret_cast<uint64_t*>(ab_smem + AbWeightBytes(G, D, Ep));
  bf16* xs = reinterpret_cast<bf16*>(ab_smem + AbWeightBytes(G, D, Ep) + 64);  // [nkb * 64] bf16 residual row
  float* sraw = reinterpret_cast<float*>(xs + nkb * 64);             // [(G + 2) d] projections before the norm
  float* sq = sraw + nout;                                           // [G][D] q after RoPE, pre-scaled
  bf16* knew = reinterpret_cast<bf16*>(sq + GD);                     // [D] this step's K row (bf16, as cached)
  bf16* vnew = knew + D;                                             // [D]
  float* wo = reinterpret_cast<float*>(vnew + D);                    // [NW][G][D]
  float* wm = wo + NW * GD;                                          // [NW][G]
  float* wl = wm + NW * G;                                           // [NW][G]
  float* sctx = wl + NW * G;                                         // [G][D] merged context
  float* srope = sctx + GD;                                          // [2][D/2] cos, sin at position p
  float* spart = srope + D;                                          // [E] this kv head's output-projection share
  const int g = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ck = lane % C, rg = lane / C;

  if (threadIdx.x == 0) {
    MbarInit(&bar[0], 1);
    FenceMbarInit();
    PrefetchTmaDesc(&tmap_qkv);
    // this kv head's rows of w_qkv: q heads g*G .. g*G+G-1, k head g, v head g, as d-row boxes
    MbarArriveExpectTx(&bar[0], (uint32_t)AbWeightBytes(G, D, Ep));
    for (int grp = 0; grp < G + 2; grp++) {
      const int row0 = grp < G ? (g * G + grp) * D : (grp == G ? (ab.H + g) * D : (ab.H + ab.Hk + g) * D);
      for (int kb = 0; kb < nkb; kb++)
        TmaLoad2D(sw + (size_t)(grp * nkb + kb) * D * 128, &tmap_qkv, &bar[0], kb * 64, row0);
    }
  }
  __syncthreads();  // barrier initialisation visible to every waiting thread

  // ---- cached K/V rows of positions 0 .. p-1 (read ahead of the wait unless the predecessor writes p) --
  int p = 0, slot = 0, ntask = 0;
  bf16* kdst = nullptr;  // the K row of position p in its page (the V row follows one K block later)
  const size_t head_off = (size_t)((ab.layer * ab.Hk + g) * 2) * kPageTokens * D;
  auto task_base = [&](int c) -> const bf16* {
    const int page = __ldcg(ab.kv.block_table + (size_t)slot * ab.kv.max_blocks + (c * kAttnTask) / kPageTokens);
    if (page < 0) {
      atomicCAS(&g_shahd_device_error, 0, kDevErrNoPage);
      return nullptr;
    }
    return ab.kv.pool + (size_t)page * ab.kv.page_elems + head_off + (size_t)((c * kAttnTask) % kPageTokens) * D;
  };
  uint4 kr[C], vr[C];  // chunk ck of rows i*RPI + rg of the warp's current task
#pragma unroll
  for (int i = 0; i < C; i++) kr[i] = vr[i] = make_uint4(0, 0, 0, 0);
  auto load_rows = [&](const bf16* kb, int c, int hi) {  // rows of task c below position hi
    const int t0 = c * kAttnTask;
    const uint4* kp = reinterpret_cast<const uint4*>(kb) + ck;
    const uint4* vp = reinterpret_cast<const uint4*>(kb + (size_t)kPageTokens * D) + ck;
#pragma unroll
    for (int i = 0; i < C; i++) {
      const int r = i * RPI + rg;
      if (t0 + r < hi) {
        kr[i] = __ldcg(kp + (size_t)r * C);
        vr[i] = __ldcg(vp + (size_t)r * C);
      }
    }
  };
  int c = warp;
  const bf16* kb = nullptr;
  auto read_ahead = [&]() {
    p = __ldcg(ab.pos + m);
    slot = __ldcg(ab.slot + m);
    ntask = p / kAttnTask + 1;
    const long long off = ab.kv.Offset(slot, p, ab.layer, g, 0);
    kdst = off >= 0 ? ab.kv.pool + off : nullptr;
    kb = c < ntask ? task_base(c) : nullptr;
    if (kb) load_rows(kb, c, p);
    for (int cc = c + NW; cc < ntask; cc += NW) {  // the warp's later tasks: into L2
      const bf16* b = task_base(cc);
      if (b) {
        for (int i = lane; i < kAttnTask * D * 2 / 128; i += 32) {
          PrefetchL2(reinterpret_cast<const char*>(b) + (size_t)i * 128);
          PrefetchL2(reinterpret_cast<const char*>(b + (size_t)kPageTokens * D) + (size_t)i * 128);
        }
      }
    }
    if (ab.rope_cos != nullptr && threadIdx.x < D)  // the RoPE row of position p, for the projection epilogue
      srope[threadIdx.x] =
          __ldg((threadIdx.x < D / 2 ? ab.rope_cos : ab.rope_sin) + (size_t)p * (D / 2) + threadIdx.x % (D / 2));
  };
  if (ab.early) read_ahead();

  GridDepWait();
  GridDepLaunch();
  if (!ab.early) read_ahead();

  // ---- norm statistics of the row's fp32 residual (every warp, from registers); warp 0 stages it as bf16 ----
  const int nch = E / 8;  // 8-float chunks of the row; lane holds chunks lane and lane + 32
  float xv[2][8];
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int ch = lane + 32 * j;
#pragma unroll
    for (int k = 0; k < 8; k++) xv[j][k] = 0.f;
    if (ch < nch) {
      const float4* src = reinterpret_cast<const float4*>(ab.x + (size_t)m * E) + 2 * ch;
      const float4 a = __ldcg(src), b = __ldcg(src + 1);
      xv[j][0] = a.x; xv[j][1] = a.y; xv[j][2] = a.z; xv[j][3] = a.w;
      xv[j][4] = b.x; xv[j][5] = b.y; xv[j][6] = b.z; xv[j][7] = b.w;
    }
  }
  if (warp == 0) {
    for (int ch = lane; ch < nkb * 8; ch += 32) {  // 16-byte pieces; zeros past E
      float f[8];
#pragma unroll
      for (int k = 0; k < 8; k++) f[k] = 0.f;
#pragma unroll
      for (int j = 0; j < 2; j++)
        if (ch == lane + 32 * j && ch < nch)
#pragma unroll
          for (int k = 0; k < 8; k++) f[k] = xv[j][k];
      StoreNbf<8>(xs + 8 * ch, f);
    }
  }
  float mu = 0.f, is;
  {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
      for (int k = 0; k < 8; k++) s += xv[j][k];
    if (ab.norm == kNormLayer) mu = WarpSum(s) / E;
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
      for (int k = 0; k < 8; k++)
        if (lane + 32 * j < nch) {
          const float dlt = xv[j][k] - mu;
          v += dlt * dlt;
        }
    is = 1.0f / sqrtf(WarpSum(v) / E + ab.eps);  // RMSNorm: mean square (mu = 0); LayerNorm: variance
  }

  // ---- Q/K/V projections of the row on the tensor cores: per 16-row tile of the staged weights, mma
  // m16n8k16 with the row as column 0 of B (lanes 0-3 carry it); two tiles per warp in flight ----
  bool ok = MbarWaitBounded(&bar[0], 0, kWaitLimit);
  if (!ok && threadIdx.x == 0) atomicCAS(&g_shahd_device_error, 0, kDevErrAttnTimeout);
  __syncthreads();  // the bf16 row and the RoPE row are in shared memory
  {
    const int ntile = nout / 16;
    const int ta = warp, tb = warp + NW;
    const bool has_a = ta < ntile, has_b = tb < ntile;
    float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
    const int mi = lane >> 3, ri = lane & 7;  // ldmatrix: this lane's matrix and row within it
    auto tile_addr = [&](int t, int kbk, int kk) -> uint32_t {
      const int r = t * 16 + ri + (mi & 1) * 8;  // weight row within the (G + 2) d rows
      const int grp = r / D, rr = r % D;
      return SmemAddr(sw + (size_t)(grp * nkb + kbk) * D * 128 + Sw128Offset(rr, kk / 8 + (mi >> 1)));
    };
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(xs);
    if (has_a) {
      for (int kbk = 0; kbk < nkb; kbk++) {
#pragma unroll
        for (int kk = 0; kk < 64; kk += 16) {
          const int k0 = kbk * 64 + kk;
          uint32_t b0 = 0u, b1 = 0u;
          if (lane < 4) {
            b0 = x32[(k0 >> 1) + lane];
            b1 = x32[(k0 >> 1) + 4 + lane];
          }
          uint32_t a[4];
          LdMatrixX4(a, tile_addr(ta, kbk, kk));
          MmaBf16_16816(da, a, b0, b1);
          if (has_b) {
            LdMatrixX4(a, tile_addr(tb, kbk, kk));
            MmaBf16_16816(db, a, b0, b1);
          }
        }
      }
      if ((lane & 3) == 0) {  // column 0 of D: rows lane/4 and lane/4 + 8 of the tile
        sraw[ta * 16 + (lane >> 2)] = da[0];
        sraw[ta * 16 + (lane >> 2) + 8] = da[2];
        if (has_b) {
          sraw[tb * 16 + (lane >> 2)] = db[0];
          sraw[tb * 16 + (lane >> 2) + 8] = db[2];
        }
      }
    }
  }
  __syncthreads();
  // epilogue per output: norm, RoPE on q and k (pairs (2i, 2i+1)), q to shared memory, k/v to the cache
  auto normed = [&](int n) -> float {
    const float acc = sraw[n];
    if (ab.norm != kNormLayer) return is * acc;
    const int col =
        n < GD ? g * GD + n : (n < GD + D ? (ab.H + g) * D + (n - GD) : (ab.H + ab.Hk + g) * D + (n - GD - D));
    return is * (acc - mu * __ldg(ab.c1 + col)) + __ldg(ab.c2 + col);
  };
  for (int n = threadIdx.x; n < nout; n += blockDim.x) {
    float v = normed(n);
    const int j = n < GD ? n % D : (n < GD + D ? n - GD : n - GD - D);
    if (ab.rope_cos != nullptr && n < GD + D) {
      const float partner = normed(n ^ 1);
      const float cs = srope[j >> 1], sn = srope[D / 2 + (j >> 1)];
      v = (j & 1) ? partner * sn + v * cs : v * cs - partner * sn;
    }
    if (n < GD) {
      sq[n] = v * ab.scale;
    } else {
      const int kvsel = n < GD + D ? 0 : 1;
      const bf16 h = __float2bfloat16_rn(v);
      (kvsel ? vnew : knew)[j] = h;
      if (kdst) kdst[(size_t)kvsel * kPageTokens * D + j] = h;
    }
  }
  __syncthreads();  // q and the new K/V row published; every warp is done with the QKV boxes

  // ---- the Wo columns of this head group into the freed buffer (16-byte asynchronous copies of every
  // thread, in flight while the attention runs) ----
  bf16* swo = reinterpret_cast<bf16*>(sw);
  {
    const int segs = GD / 8;  // 16-byte pieces per Wo row segment
    for (int i = threadIdx.x; i < E * segs; i += blockDim.x) {
      const int e = i / segs, sg = i - e * segs;
      CpAsync16(swo + (size_t)e * GD + 8 * sg, ab.w_o + (size_t)e * ab.HDp + (size_t)g * GD + 8 * sg);
    }
    CpAsyncCommit();
  }

  // ---- attention over positions 0 .. p (the row at p from shared memory) ----
  auto take_new_row = [&](int cc) {
    const int t0 = cc * kAttnTask;
#pragma unroll
    for (int i = 0; i < C; i++)
      if (t0 + i * RPI + rg == p) {
        kr[i] = reinterpret_cast<const uint4*>(knew)[ck];
        vr[i] = reinterpret_cast<const uint4*>(vnew)[ck];
      }
  };
  float o[MG][8], mrun[MG], lrun[MG];
#pragma unroll
  for (int h = 0; h < MG; h++) {
    mrun[h] = -INFINITY;
    lrun[h] = 0.f;
#pragma unroll
    for (int jj = 0; jj < 8; jj++) o[h][jj] = 0.f;
  }
  for (bool first = true; c < ntask; c += NW, first = false) {
    const int t0 = c * kAttnTask;
    if (!first) {
      kb = task_base(c);
#pragma unroll
      for (int i = 0; i < C; i++) kr[i] = vr[i] = make_uint4(0, 0, 0, 0);  // rows past p stay zero
      if (kb) load_rows(kb, c, p);
    }
    if (kb == nullptr) continue;  // missing page: its positions are left out (the error flag is set)
    take_new_row(c);
    const bool valid = t0 + ck * RPI + rg <= p;  // the row this lane scores
    float pv[MG];
#pragma unroll
    for (int h = 0; h < MG; h++) {
      pv[h] = 0.f;
      if (h < G) {
        const float4 q0 = *reinterpret_cast<const float4*>(sq + h * D + ck * 8);
        const float4 q1 = *reinterpret_cast<const float4*>(sq + h * D + ck * 8 + 4);
        const float qf[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        float sc_part[C];
#pragma unroll
        for (int i = 0; i < C; i++) {
          float kf[8];
          Bf16ChunkToFloat(kr[i], kf);
          float a = 0.f;
#pragma unroll
          for (int jj = 0; jj < 8; jj++) a = fmaf(qf[jj], kf[jj], a);
          sc_part[i] = a;
        }
        const float full = ReduceScatter<C>(sc_part, lane);  // every lane takes part in the shuffles
        const float si = valid ? full : -INFINITY;
        const float nm = fmaxf(mrun[h], WarpMax(si));
        const float sc = mrun[h] == -INFINITY ? 0.f : __expf(mrun[h] - nm);
        pv[h] = valid ? __expf(si - nm) : 0.f;
        lrun[h] = lrun[h] * sc + pv[h];
#pragma unroll
        for (int jj = 0; jj < 8; jj++) o[h][jj] *= sc;
        mrun[h] = nm;
      }
    }
#pragma unroll
    for (int i = 0; i < C; i++) {
      float vf[8];
      Bf16ChunkToFloat(vr[i], vf);
#pragma unroll
      for (int h = 0; h < MG; h++) {
        if (h < G) {
          const float pt = __shfl_sync(0xffffffffu, pv[h], rg * C + i);
#pragma unroll
          for (int jj = 0; jj < 8; jj++) o[h][jj] = fmaf(pt, vf[jj], o[h][jj]);
        }
      }
    }
  }
#pragma unroll
  for (int h = 0; h < MG; h++) {
    if (h < G) {
#pragma unroll
      for (int jj = 0; jj < 8; jj++)
#pragma unroll
        for (int off = C; off < 32; off *= 2) o[h][jj] += __shfl_xor_sync(0xffffffffu, o[h][jj], off);
      const float l = WarpSum(lrun[h]);
      if (lane == 0) {
        wm[warp * G + h] = mrun[h];
        wl[warp * G + h] = l;
      }
      if (rg == 0) {
#pragma unroll
        for (int jj = 0; jj < 8; jj++) wo[(warp * G + h) * D + ck * 8 + jj] = o[h][jj];
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < GD; e += blockDim.x) {  // merge the warps (idle warps: max = -inf)
    const int i = e / D;
    float M = -INFINITY, L = 0.f, acc = 0.f;
    for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w * G + i]);
    for (int w = 0; w < NW; w++)
      if (wm[w * G + i] != -INFINITY) {
        const float f = __expf(wm[w * G + i] - M);
        L += f * wl[w * G + i];
        acc += f * wo[(w * G + i) * D + e % D];
      }
    sctx[e] = acc / L;
  }
  CpAsyncWaitAll();
  __syncthreads();  // the merged context and every thread's Wo pieces are in shared memory

  // ---- this head group's share of the output projection: spart = ctx_g . Wo[:, g]^T ----
  const int nco = GD / 8;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const bf16* wrow = swo + (size_t)e * GD;
    float acc = 0.f;
    for (int cc = 0; cc < nco; cc++) {
      const int ch = (cc + e) % nco;  // rotated chunk order: the lanes of a quarter-warp hit distinct banks
      float wf[8];
      Bf16ChunkToFloat(*reinterpret_cast<const uint4*>(wrow + 8 * ch), wf);
      const float4 c0 = *reinterpret_cast<const float4*>(sctx + 8 * ch);
      const float4 c1v = *reinterpret_cast<const float4*>(sctx + 8 * ch + 4);
      acc = fmaf(wf[0], c0.x, acc);
      acc = fmaf(wf[1], c0.y, acc);
      acc = fmaf(wf[2], c0.z, acc);
      acc = fmaf(wf[3], c0.w, acc);
      acc = fmaf(wf[4], c1v.x, acc);
      acc = fmaf(wf[5], c1v.y, acc);
      acc = fmaf(wf[6], c1v.z, acc);
      acc = fmaf(wf[7], c1v.w, acc);
    }
    spart[e] = acc;
  }
  // ---- the row's kv heads form a cluster: its first CTA adds their shares to the residual in kv-head order
  // (CachedForward.ts:81-84), reading them from the peers' shared memory ----
  ClusterSync();
  if (ClusterCtaRank() == 0) {
    for (int e4 = threadIdx.x; e4 < E / 4; e4 += blockDim.x) {
      float4 v = *reinterpret_cast<const float4*>(ab.x + (size_t)m * E + 4 * e4);
      for (int r = 0; r < ab.Hk; r++) {
        const float4 t = LoadPeerF32x4(spart + 4 * e4, (uint32_t)r);
        v.x += t.x;
        v.y += t.y;
        v.z += t.z;
        v.w += t.w;
      }
      *reinterpret_cast<float4*>(ab.x + (size_t)m * E + 4 * e4) = v;
      const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; k++) ab.xb[(size_t)m * ab.ldxb + 4 * e4 + k] = __float2bfloat16_rn(f[k]);
    }
  }
  ClusterSync();  // the peers keep their shares until the first CTA has read them
  if (!ok && threadIdx.x == 0) {
    // a weight copy that timed out may still land: let it finish (bounded) before the shared memory goes
    MbarWaitBounded(&bar[0], 0, kWaitLimit);
  }
}

extern int g_fused_attn_block;

// Two CTAs per SM must fit (the grid is rows x kv heads, at least one wave), the warps hold the residual
// row in registers, the projection outputs come in whole 16-row tiles (at most two per warp), the Wo
// columns fit in the freed weight buffer and a row's kv heads form one portable cluster.
constexpr int kAbMaxSmem = 110 * 1024;
inline bool AttnBlockFits(int d, int G, int Hk, int E, int Ep) {
  return (d == 32 || d == 64) && G >= 1 && G <= 4 && Hk >= 1 && Hk <= 8 && E % 8 == 0 && E <= kAbMaxE &&
         Ep % 8 == 0 && Ep >= 64 && (G + 2) * d <= 2 * 16 * kAbWarps && AbSmemBytes(G, d, Ep) <= kAbMaxSmem &&
         E * G * d * 2 <= AbWeightBytes(G, d, Ep);
}

template <int D>
inline bool EnsureAttnBlockAttrsD(int G, int Ep) {
  const int sm = AbSmemBytes(G, D, Ep);
  if (G == 1) return EnsureKernelAttrs((const void*)AttnBlockKernel<D, 1>, sm);
  if (G == 2) return EnsureKernelAttrs((const void*)AttnBlockKernel<D, 2>, sm);
  return EnsureKernelAttrs((const void*)AttnBlockKernel<D, 4>, sm);
}
inline bool EnsureAttnBlockAttrs(int d, int G, int Ep) {
  return d == 64 ? EnsureAttnBlockAttrsD<64>(G, Ep) : EnsureAttnBlockAttrsD<32>(G, Ep);
}

// Grid (1, kv heads, rows) in clusters of the row's kv heads; the Q/K/V weights of the layer
// ([(H + 2 Hk) d, Ep] bf16) through a TMA map of d-row boxes.
template <int D>
inline void LaunchAttnBlockD(const AttnBlockArgs& ab, const CUtensorMap& tm, int M, cudaStream_t st) {
  const dim3 grid(1, ab.Hk, M), cluster(1, ab.Hk, 1);
  const int sm = AbSmemBytes(ab.G, D, ab.Ep);
  if (ab.G == 1) LaunchPdlCluster(AttnBlockKernel<D, 1>, grid, dim3(kAbThreads), sm, cluster, st, ab, tm);
  else if (ab.G == 2) LaunchPdlCluster(AttnBlockKernel<D, 2>, grid, dim3(kAbThreads), sm, cluster, st, ab, tm);
  else LaunchPdlCluster(AttnBlockKernel<D, 4>, grid, dim3(kAbThreads), sm, cluster, st, ab, tm);
}
inline void LaunchAttnBlock(int d, const AttnBlockArgs& ab, const bf16* w_qkv, int nqkv, int M, cudaStream_t st) {
  CUtensorMap tm;
  if (!MakeTmaBf16(w_qkv, nqkv, ab.Ep, ab.Ep, d, &tm)) {
    NoteLaunchError(cudaErrorInvalidValue, "cuTensorMapEncodeTiled for the fused attention block");
    return;
  }
  if (d == 64) LaunchAttnBlockD<64>(ab, tm, M, st);
  else LaunchAttnBlockD<32>(ab, tm, M, st);
}

}  // namespace shahd
