// Seeded stochastic token selection on the device: SampleFromLogits with Temperature > 0
// (Brain/Sampling/Sampler.ts:16-27) = ProbsFromLogits (temperature softmax, top-k, top-p over the
// renormalized top-k mass; Distribution.ts:35-89) + SampleFromDistribution (one SeededRng draw, inverse
// CDF in ascending index order; Distribution.ts:93-104) for every decode row at once.
//
// The reference sorts the whole vocabulary; here the kept set is found without sorting. The sorted order
// (probability descending, index ascending: a stable sort of Probs[B] - Probs[A]) is a total order on
// (key, index) with key = the fp32 bits of exp(l/T - max), which are ordered like the values because the
// values are >= 0. A most-significant-digit radix descent over the key (four 8-bit digits) finds the
// k-th key for top-k and the key at which the running mass reaches TopP of the kept mass for top-p; ties at
// that key are taken in ascending index order, as the stable sort takes them.
//
// Masses are fixed point: m = round(e * 2^40) as u64 (e <= 1, V <= 2^22 keeps every sum below 2^63), so
// every sum is exact and the kept set and the drawn id do not depend on the order of the additions.
// The inverse CDF compares cum * 2^32 >= draw * KeptSum in 128 bits, with u = draw / 2^32 exactly as
// SeededRng.NextFloat (SeededRng.ts:32-40) makes it.
#pragma once

#include "common.cuh"

namespace shahd {

constexpr int kSampleThreads = 1024;
constexpr double kMassScale = 1099511627776.0;  // 2^40

struct SampleArgs {
  float* probs;        // [M, V]: the row's logits in; overwritten with exp(l/T - max)
  int V;
  const int* slot;     // [M]
  uint32_t* rng;       // [max_seqs] SeededRng state per slot, advanced once per sampled row
  float temperature;   // <= 0: greedy argmax, no draw
  int top_k;           // <= 0 or >= V: disabled
  double top_p;        // >= 1: disabled
  int* sampled;        // [M] chosen ids
};

namespace sample_detail {

struct Shared {
  unsigned long long mass[256];
  int cnt[256];
  unsigned long long warp_u64[32];
  float warp_f[32];
  int warp_i[32];
  unsigned long long total;
  int sel, rem, tie_idx, ans, last_nz;
  unsigned long long mass_above;
  uint32_t draw;
};

__device__ __forceinline__ float BlockMax(float v, Shared& sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) sh.warp_f[w] = v;
  __syncthreads();
  float r = -INFINITY;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) r = fmaxf(r, sh.warp_f[i]);
  __syncthreads();
  return r;
}

// Exclusive prefix over threads in index order (u64); also returns the block total.
__device__ __forceinline__ unsigned long long BlockExclusiveU64(unsigned long long v, unsigned long long* total,
                                                               Shared& sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  unsigned long long incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) sh.warp_u64[w] = incl;
  __syncthreads();
  unsigned long long before = 0, all = 0;
  for (int i = 0; i < nw; i++) {
    if (i < w) before += sh.warp_u64[i];
    all += sh.warp_u64[i];
  }
  __syncthreads();
  *total = all;
  return before + incl - v;
}

__device__ __forceinline__ int BlockExclusiveInt(int v, int* total, Shared& sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) sh.warp_i[w] = incl;
  __syncthreads();
  int before = 0, all = 0;
  for (int i = 0; i < nw; i++) {
    if (i < w) before += sh.warp_i[i];
    all += sh.warp_i[i];
  }
  __syncthreads();
  *total = all;
  return before + incl - v;
}

__device__ __forceinline__ unsigned long long Mass(float e) { return __double2ull_rn((double)e * kMassScale); }

// (key, index) strictly after the cut (k, i) in the sorted order, or the cut itself: the kept prefix.
__device__ __forceinline__ bool InPrefix(uint32_t key, int j, uint32_t cut_key, int cut_idx) {
  return key > cut_key || (key == cut_key && j <= cut_idx);
}

__device__ __forceinline__ bool DigitMatch(uint32_t key, uint32_t prefix, int shift) {
  return shift == 24 || (key >> (shift + 8)) == (prefix >> (shift + 8));
}

// Index of the tie with rank `rank` (0-based, ascending index) among elements of this thread's chunk that
// satisfy `is_tie`, written to sh.tie_idx by the owning thread; sh.tie_idx must be preset.
template <class P>
__device__ __forceinline__ void FindTie(int j0, int j1, int rank, P is_tie, Shared& sh) {
  int mine = 0;
  for (int j = j0; j < j1; j++) mine += is_tie(j) ? 1 : 0;
  int total;
  const int before = BlockExclusiveInt(mine, &total, sh);
  if (rank >= total) rank = total - 1;  // fewer ties than asked for: the last one
  if (rank >= before && rank < before + mine) {
    int r = before;
    for (int j = j0; j < j1; j++)
      if (is_tie(j)) {
        if (r == rank) {
          sh.tie_idx = j;
          break;
        }
        r++;
      }
  }
  __syncthreads();
}

// The kept set of ProbsFromLogits (Distribution.ts:35-89) over one row: the row's logits become the
// temperature-softmax numerators exp(l/T - max) in place, and the kept set is the prefix of the sorted order
// up to (cut_key, cut_idx), with kept_sum the fixed-point mass of the whole kept set. Probability of a kept j:
// Mass(row[j]) / kept_sum. Called by every thread of the block (T > 0).
struct KeptSet {
  uint32_t cut_key;
  int cut_idx;
  unsigned long long kept_sum;
};

__device__ __forceinline__ bool Kept(const float* row, int j, const KeptSet& k) {
  return InPrefix(__float_as_uint(row[j]), j, k.cut_key, k.cut_idx);
}
__device__ __forceinline__ double KeptProb(const float* row, int j, const KeptSet& k) {
  return Kept(row, j, k) && k.kept_sum > 0 ? (double)Mass(row[j]) / (double)k.kept_sum : 0.0;
}

__device__ KeptSet ComputeKept(float* row, int V, float temperature, int top_k, double top_p, Shared& sh) {
  const int chunk = CeilDiv(V, (int)blockDim.x);
  const int j0 = min(V, (int)threadIdx.x * chunk), j1 = min(V, j0 + chunk);
  // temperature softmax numerators (Distribution.ts:41-55); each thread touches only its own chunk
  float mx = -INFINITY;
  for (int j = j0; j < j1; j++) mx = fmaxf(mx, row[j] / temperature);
  mx = BlockMax(mx, sh);
  for (int j = j0; j < j1; j++) row[j] = expf(row[j] / temperature - mx);

  // kept set = prefix of the sorted order up to the cut (cut_key, cut_idx); everything to start with
  uint32_t cut_key = 0;
  int cut_idx = V - 1;

  // top-k (Distribution.ts:68): the k-th (key, index) of the sorted order
  if (top_k > 0 && top_k < V) {
    uint32_t prefix = 0;
    int remaining = top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) sh.cnt[b] = 0;
      __syncthreads();
      for (int j = j0; j < j1; j++) {
        const uint32_t key = __float_as_uint(row[j]);
        if (DigitMatch(key, prefix, shift)) atomicAdd(&sh.cnt[(key >> shift) & 255], 1);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int b = 255;
        for (; b > 0; b--) {
          if (sh.cnt[b] >= remaining) break;
          remaining -= sh.cnt[b];
        }
        sh.sel = b;
        sh.rem = remaining;
      }
      __syncthreads();
      prefix |= (uint32_t)sh.sel << shift;
      remaining = sh.rem;
      __syncthreads();
    }
    // `remaining` ties at key == prefix are kept, lowest indices first (the stable sort's order)
    if (threadIdx.x == 0) sh.tie_idx = V - 1;
    __syncthreads();
    const uint32_t kk = prefix;
    FindTie(j0, j1, remaining - 1, [&](int j) { return __float_as_uint(row[j]) == kk; }, sh);
    cut_key = kk;
    cut_idx = sh.tie_idx;
  }

  // top-p over the renormalized top-k mass (Distribution.ts:69-82): the first (key, index) at which the
  // running mass reaches TopP * TopKMass
  if (top_p < 1.0) {
    unsigned long long mine = 0, topk_mass;
    for (int j = j0; j < j1; j++)
      if (InPrefix(__float_as_uint(row[j]), j, cut_key, cut_idx)) mine += Mass(row[j]);
    BlockExclusiveU64(mine, &topk_mass, sh);
    const double tp = top_p > 0.0 ? top_p : 0.0;
    const unsigned long long thr = (unsigned long long)ceil(tp * (double)topk_mass);
    uint32_t prefix = 0;
    unsigned long long above = 0;  // mass of kept elements with a larger key than the digits chosen so far
    bool found_all = true;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) {
        sh.cnt[b] = 0;
        sh.mass[b] = 0;
      }
      __syncthreads();
      for (int j = j0; j < j1; j++) {
        const uint32_t key = __float_as_uint(row[j]);
        if (InPrefix(key, j, cut_key, cut_idx) && DigitMatch(key, prefix, shift)) {
          atomicAdd(&sh.cnt[(key >> shift) & 255], 1);
          atomicAdd(&sh.mass[(key >> shift) & 255], Mass(row[j]));
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int sel = -1, lowest = -1;
        unsigned long long acc = above, acc_at_lowest = above;
        for (int b = 255; b >= 0; b--) {
          if (sh.cnt[b] == 0) continue;
          if (acc + sh.mass[b] >= thr) {
            sel = b;
            break;
          }
          acc_at_lowest = acc;
          lowest = b;
          acc += sh.mass[b];
        }
        // rounding can leave the threshold above the whole kept mass: then everything stays
        sh.rem = sel >= 0 ? 1 : 0;
        sh.sel = sel >= 0 ? sel : lowest;
        sh.mass_above = sel >= 0 ? acc : acc_at_lowest;
      }
      __syncthreads();
      if (!sh.rem) found_all = false;
      prefix |= (uint32_t)sh.sel << shift;
      above = sh.mass_above;
      __syncthreads();
      if (!found_all) break;
    }
    if (found_all) {
      // ties at the cut key in ascending index order: the first n with above + n * m >= thr (n >= 1)
      const uint32_t pk = prefix;
      const unsigned long long mt = Mass(__uint_as_float(pk));
      const unsigned long long gap = thr > above ? thr - above : 0;
      long long n = mt > 0 ? (long long)((gap + mt - 1) / mt) : 1;
      if (n < 1) n = 1;
      if (n > V) n = V;
      if (threadIdx.x == 0) sh.tie_idx = V - 1;
      __syncthreads();
      const uint32_t ck = cut_key;
      const int ci = cut_idx;
      FindTie(j0, j1, (int)(n - 1),
              [&](int j) {
                const uint32_t key = __float_as_uint(row[j]);
                return key == pk && InPrefix(key, j, ck, ci);
              },
              sh);
      // the top-p cut lies inside the top-k prefix, so it replaces it
      cut_key = pk;
      cut_idx = sh.tie_idx;
    }
  }

  KeptSet k{cut_key, cut_idx, 0};
  unsigned long long mine = 0;
  for (int j = j0; j < j1; j++)
    if (InPrefix(__float_as_uint(row[j]), j, cut_key, cut_idx)) mine += Mass(row[j]);
  BlockExclusiveU64(mine, &k.kept_sum, sh);
  return k;
}

// SampleFromDistribution (Distribution.ts:93-104) over a kept set with the draw `draw` (u = draw / 2^32): the
// first kept j with a nonzero mass whose running mass reaches u * kept_sum, else the last such j, else 0.
// Returns the id in every thread.
__device__ int DrawKept(const float* row, int V, const KeptSet& ks, uint32_t draw_u32, Shared& sh) {
  const int chunk = CeilDiv(V, (int)blockDim.x);
  const int j0 = min(V, (int)threadIdx.x * chunk), j1 = min(V, j0 + chunk);
  const uint32_t cut_key = ks.cut_key;
  const int cut_idx = ks.cut_idx;
  if (threadIdx.x == 0) {
    sh.ans = -1;
    sh.last_nz = -1;
  }
  __syncthreads();
  // inverse CDF in ascending index order over the kept set (Distribution.ts:84-104): the first kept j with
  // m_j > 0 and cum_j >= u * KeptSum, u = draw / 2^32
  unsigned long long mine = 0, kept_sum;
  for (int j = j0; j < j1; j++)
    if (InPrefix(__float_as_uint(row[j]), j, cut_key, cut_idx)) mine += Mass(row[j]);
  const unsigned long long before = BlockExclusiveU64(mine, &kept_sum, sh);
  const uint64_t draw = draw_u32;
  const unsigned long long t_lo = draw * kept_sum, t_hi = __umul64hi(draw, kept_sum);
  auto reaches = [&](unsigned long long cum) {  // cum * 2^32 >= draw * kept_sum
    const unsigned long long c_hi = cum >> 32, c_lo = cum << 32;
    return c_hi > t_hi || (c_hi == t_hi && c_lo >= t_lo);
  };
  if (mine > 0 && reaches(before + mine) && (before == 0 || !reaches(before))) {
    unsigned long long cum = before;
    for (int j = j0; j < j1; j++) {
      const float e = row[j];
      if (!InPrefix(__float_as_uint(e), j, cut_key, cut_idx)) continue;
      const unsigned long long m = Mass(e);
      if (m == 0) continue;
      cum += m;
      if (reaches(cum)) {
        sh.ans = j;
        break;
      }
    }
  }
  if (mine > 0) {
    int last = -1;
    for (int j = j0; j < j1; j++)
      if (InPrefix(__float_as_uint(row[j]), j, cut_key, cut_idx) && Mass(row[j]) > 0) last = j;
    atomicMax(&sh.last_nz, last);
  }
  __syncthreads();
  int id = sh.ans;
  if (id < 0) id = sh.last_nz >= 0 ? sh.last_nz : 0;  // SampleFromDistribution's fallbacks
  __syncthreads();
  return id;
}

}  // namespace sample_detail

__global__ void __launch_bounds__(kSampleThreads) SampleKernel(SampleArgs a) {
  using namespace sample_detail;
  __shared__ Shared sh;
  GridDepWait();
  GridDepLaunch();
  const int r = blockIdx.x;
  const int V = a.V;
  float* row = a.probs + (size_t)r * V;
  const int chunk = CeilDiv(V, (int)blockDim.x);
  const int j0 = min(V, (int)threadIdx.x * chunk), j1 = min(V, j0 + chunk);
  if (!(a.temperature > 0)) {
    // Temperature <= 0: ArgmaxOf (Distribution.ts:19-30), the first index of the strict max; no draw
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = j0; j < j1; j++) ArgmaxMerge(bv, bi, row[j], j);
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      ArgmaxMerge(bv, bi, ov, oi);
    }
    if ((threadIdx.x & 31) == 0) {
      sh.warp_f[threadIdx.x >> 5] = bv;
      sh.warp_i[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); w++) ArgmaxMerge(bv, bi, sh.warp_f[w], sh.warp_i[w]);
      a.sampled[r] = bi == 0x7fffffff ? 0 : bi;
    }
    return;
  }
  if (threadIdx.x == 0) {
    uint32_t* st = a.rng + a.slot[r];
    const uint32_t next = *st * 1664525u + 1013904223u;  // SeededRng.NextUint32 (SeededRng.ts:32-35)
    *st = next;
    sh.draw = next;
  }
  const KeptSet ks = ComputeKept(row, V, a.temperature, a.top_k, a.top_p, sh);
  const int id = DrawKept(row, V, ks, sh.draw, sh);
  if (threadIdx.x == 0) a.sampled[r] = id;
}

}  // namespace shahd

namespace shahd {

// ---- one verification round of stochastic speculative sampling on the device ------------------------------
// SpeculativeSample (Brain/Reasoning/SpeculativeSampling.ts:82-112) for many sequences at once, one CTA each:
// proposal i is accepted with probability min(1, p/q) (one SeededRng draw per examined proposal); the first
// rejection is replaced by a draw from the normalized residual max(0, p - q) (ResidualSample, :23-36; from p
// when the residual has no mass); when every proposal is accepted and budget is left, a bonus id is drawn
// from the target's distribution after the last proposal. p and q are ProbsFromLogits of the target and draft
// rows (the kept sets of the sampler above, fixed-point masses); the acceptance test and the residual walk
// run in fp64 like the reference's Float64Array arithmetic.

struct SpecArgs {
  float* target;          // [n][gmax + 1][V] logits (overwritten with softmax numerators)
  float* draft;           // [n][gmax][V] logits of the distributions the proposals were drawn from
  const int* proposals;   // [n][gmax]
  const int* g;           // [n] proposals of each sequence this round
  const int* budget;      // [n] new ids each sequence may still take
  int gmax, V;
  uint32_t* rng;          // [n] SeededRng state of each sequence, advanced in place
  float temperature;
  int top_k;
  double top_p;
  int* out;               // [n][gmax + 1] appended ids
  int* count;             // [n] ids appended
  int* accepted;          // [n] proposals accepted
};

namespace sample_detail {

struct SpecShared {
  double warp_d[32];
  int accept, ans, last_nz;
};

__device__ __forceinline__ uint32_t NextDraw(uint32_t* st) {
  const uint32_t next = *st * 1664525u + 1013904223u;  // SeededRng.NextUint32 (SeededRng.ts:32-35)
  *st = next;
  return next;
}

// Exclusive prefix (index order of threads) of a double and the block total.
__device__ __forceinline__ double BlockExclusiveF64(double v, double* total, SpecShared& sp) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  double incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) sp.warp_d[w] = incl;
  __syncthreads();
  double before = 0, all = 0;
  for (int i = 0; i < nw; i++) {
    if (i < w) before += sp.warp_d[i];
    all += sp.warp_d[i];
  }
  __syncthreads();
  *total = all;
  return before + incl - v;
}

}  // namespace sample_detail

__global__ void __launch_bounds__(kSampleThreads) SpecRoundKernel(SpecArgs a) {
  using namespace sample_detail;
  __shared__ Shared sh;
  __shared__ SpecShared sp;
  const int sq = blockIdx.x, V = a.V;
  const int g = a.g[sq], budget = a.budget[sq];
  const int chunk = CeilDiv(V, (int)blockDim.x);
  const int j0 = min(V, (int)threadIdx.x * chunk), j1 = min(V, j0 + chunk);
  uint32_t* st = a.rng + sq;
  int n = 0, acc = 0;
  bool corrected = false;
  for (int i = 0; i < g && n < budget; i++) {
    float* trow = a.target + ((size_t)sq * (a.gmax + 1) + i) * V;
    float* drow = a.draft + ((size_t)sq * a.gmax + i) * V;
    const KeptSet P = ComputeKept(trow, V, a.temperature, a.top_k, a.top_p, sh);
    const KeptSet Q = ComputeKept(drow, V, a.temperature, a.top_k, a.top_p, sh);
    const int tok = a.proposals[sq * a.gmax + i];
    if (threadIdx.x == 0) {
      const double p = KeptProb(trow, tok, P), q = KeptProb(drow, tok, Q);
      const double ratio = q > 0 ? p / q : (p > 0 ? 1.0 : 0.0);
      const double u = (double)NextDraw(st) / 4294967296.0;  // SeededRng.NextFloat (SeededRng.ts:38-40)
      sp.accept = u < (ratio < 1.0 ? ratio : 1.0) ? 1 : 0;
    }
    __syncthreads();
    if (sp.accept) {
      if (threadIdx.x == 0) a.out[sq * (a.gmax + 1) + n] = tok;
      n++;
      acc++;
      __syncthreads();
      continue;
    }
    // ResidualSample: max(0, p - q) over the vocabulary, normalized by its sum, walked in index order
    double mine = 0;
    for (int j = j0; j < j1; j++) {
      const double r = KeptProb(trow, j, P) - KeptProb(drow, j, Q);
      if (r > 0) mine += r;
    }
    double sum;
    const double before = BlockExclusiveF64(mine, &sum, sp);
    int id;
    if (!(sum > 0)) {  // degenerate residual: a draw from the target's distribution
      if (threadIdx.x == 0) sh.draw = NextDraw(st);
      __syncthreads();
      id = DrawKept(trow, V, P, sh.draw, sh);
    } else {
      if (threadIdx.x == 0) {
        sh.draw = NextDraw(st);
        sp.ans = -1;
        sp.last_nz = -1;
      }
      __syncthreads();
      const double target_mass = (double)sh.draw / 4294967296.0 * sum;  // R -= r_j / sum until R <= 0
      if (mine > 0 && before + mine >= target_mass && !(before > 0 && before >= target_mass)) {
        double cum = before;
        for (int j = j0; j < j1; j++) {
          const double r = KeptProb(trow, j, P) - KeptProb(drow, j, Q);
          if (!(r > 0)) continue;
          cum += r;
          if (cum >= target_mass) {
            sp.ans = j;
            break;
          }
        }
      }
      if (mine > 0) {
        int last = -1;
        for (int j = j0; j < j1; j++)
          if (KeptProb(trow, j, P) - KeptProb(drow, j, Q) > 0) last = j;
        atomicMax(&sp.last_nz, last);
      }
      __syncthreads();
      id = sp.ans >= 0 ? sp.ans : (sp.last_nz >= 0 ? sp.last_nz : 0);
    }
    if (threadIdx.x == 0) a.out[sq * (a.gmax + 1) + n] = id;
    n++;
    corrected = true;
    __syncthreads();
    break;
  }
  if (!corrected && n < budget) {  // every proposal accepted: the bonus id from the target's own distribution
    float* trow = a.target + ((size_t)sq * (a.gmax + 1) + g) * V;
    const KeptSet P = ComputeKept(trow, V, a.temperature, a.top_k, a.top_p, sh);
    if (threadIdx.x == 0) sh.draw = NextDraw(st);
    __syncthreads();
    const int id = DrawKept(trow, V, P, sh.draw, sh);
    if (threadIdx.x == 0) a.out[sq * (a.gmax + 1) + n] = id;
    n++;
  }
  if (threadIdx.x == 0) {
    a.count[sq] = n;
    a.accepted[sq] = acc;
  }
}

}  // namespace shahd
