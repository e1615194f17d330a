// Host side of the weight boundary: the reference's flat parameter order (Shahd.Parameters(),
// Brain/Nn/Shahd.ts:87-94), its weight initialization (Shahd.ts:30-39 + InitPolicy.ts:15-24 +
// SeededRng.ts), and the repack into the device layout the kernels read:
//   w_qkv [(H + 2 Hk) d, Ep]  rows = Q heads, then K heads, then V heads (column j of each [E,d] head)
//   w_o   [E, HDp]            row e = output dim, col h*d + j = Wo_h[j, e] (per-head Wo summed = concat)
//   w_up  [2F, Ep] gated      rows 2j / 2j+1 = W1[:, j] / W3[:, j] (gate/up interleaved per column pair)
//         [F, Ep]  relu       row f = Wfc[:, f]
//   w_down [E, Fp]            row e = W2[:, e] (or Wproj)
//   w_head [V, Ep]            tied: Wte rows; untied: LmHead columns
// All bf16, reduction dims zero-padded to multiples of 8 (16-byte rows for TMA); biases, embedding
// tables and the RoPE cos/sin table stay fp32. The norm in front of w_qkv / w_up / w_head is folded in:
// those weights carry gamma (W'[n,k] = W[n,k]·gamma[k]); for LayerNorm the per-column constants
// c1[n] = sum_k W'[n,k] and c2[n] = sum_k beta[k]·W[n,k] let the kernels apply the mean and beta.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include <cmath>
#include <vector>

#include "../../include/shahd_b200.h"
#include "common.cuh"

namespace shahd {

struct LayerParamOff {
  int64_t ln1_g, ln1_b, ln2_g, ln2_b, wq, wk, wv, wo, wfc, bfc, wproj, bproj, w1, w3, w2;
};

struct ParamLayout {
  int64_t wte, wpe, lnf_g, lnf_b, lm_head, lm_bias, total;
  std::vector<LayerParamOff> layers;
};

inline int BuildParamLayout(const ShahdModelCfg& c, ParamLayout* lay) {
  if (c.embed_dim < 1 || c.num_layers < 1 || c.num_heads < 1 || c.kv_heads < 1 || c.block_size < 1 ||
      c.vocab_size < 1 || c.mlp_hidden < 1) {
    SetError("model config: every dimension must be >= 1");
    return SHAHD_EINVAL;
  }
  if (c.embed_dim % c.num_heads != 0) {
    SetError("model config: EmbedDim %d must be divisible by NumHeads %d", c.embed_dim, c.num_heads);
    return SHAHD_EINVAL;
  }
  if (c.num_heads % c.kv_heads != 0) {
    SetError("model config: NumHeads %d must be divisible by KvHeads %d", c.num_heads, c.kv_heads);
    return SHAHD_EINVAL;
  }
  if (c.position_scheme < 0 || c.position_scheme > 1 || c.norm_kind < 0 || c.norm_kind > 1 || c.mlp_kind < 0 ||
      c.mlp_kind > 2) {
    SetError("model config: position_scheme/norm_kind/mlp_kind out of range");
    return SHAHD_EINVAL;
  }
  const int64_t E = c.embed_dim, H = c.num_heads, Hk = c.kv_heads, d = E / H, F = c.mlp_hidden;
  const bool ln = c.norm_kind == 0;
  int64_t o = 0;
  lay->wte = o; o += (int64_t)c.vocab_size * E;
  lay->wpe = -1;
  if (c.position_scheme == 0) { lay->wpe = o; o += (int64_t)c.block_size * E; }
  lay->layers.assign(c.num_layers, LayerParamOff{});
  for (int l = 0; l < c.num_layers; l++) {
    LayerParamOff& L = lay->layers[l];
    L.ln1_g = o; o += E;
    L.ln1_b = -1; if (ln) { L.ln1_b = o; o += E; }
    L.wq = o; o += H * E * d;
    L.wk = o; o += Hk * E * d;
    L.wv = o; o += Hk * E * d;
    L.wo = o; o += H * d * E;
    L.ln2_g = o; o += E;
    L.ln2_b = -1; if (ln) { L.ln2_b = o; o += E; }
    L.wfc = L.bfc = L.wproj = L.bproj = L.w1 = L.w3 = L.w2 = -1;
    if (c.mlp_kind == 0) {
      L.wfc = o; o += E * F;
      L.bfc = o; o += F;
      L.wproj = o; o += F * E;
      L.bproj = o; o += E;
    } else {
      L.w1 = o; o += E * F;
      L.w3 = o; o += E * F;
      L.w2 = o; o += F * E;
    }
  }
  lay->lnf_g = o; o += E;
  lay->lnf_b = -1; if (ln) { lay->lnf_b = o; o += E; }
  lay->lm_head = -1;
  if (!c.weight_tying) { lay->lm_head = o; o += E * c.vocab_size; }
  lay->lm_bias = o; o += c.vocab_size;
  lay->total = o;
  return SHAHD_OK;
}

struct HostLayer {
  std::vector<bf16> w_qkv, w_o, w_up, w_down;
  std::vector<float> qkv_c1, qkv_c2, up_c1, up_c2, b_fc, b_proj;
};

struct HostWeights {
  std::vector<HostLayer> layers;
  std::vector<bf16> w_head;
  std::vector<float> head_bias, head_c1, head_c2, wte, wpe, rope_cos, rope_sin;
};

// Folds the norm (gamma, beta) in front of a projection stored as w [N, Kp] (rows already = columns of
// the reference [K, N] matrix, in fp32 in `wf`): w = bf16(wf * gamma); LayerNorm constants c1/c2.
inline void FoldNorm(const std::vector<float>& wf, int N, int K, int Kp, const float* gamma, const float* beta,
                     bool layer_norm, std::vector<bf16>* w, std::vector<float>* c1, std::vector<float>* c2) {
  w->assign((size_t)N * Kp, __float2bfloat16_rn(0.f));
  if (layer_norm) {
    c1->assign(N, 0.f);
    c2->assign(N, 0.f);
  }
  for (int n = 0; n < N; n++) {
    double s1 = 0, s2 = 0;
    for (int k = 0; k < K; k++) {
      const float orig = wf[(size_t)n * K + k];
      const bf16 b = __float2bfloat16_rn(orig * gamma[k]);
      (*w)[(size_t)n * Kp + k] = b;
      s1 += (double)__bfloat162float(b);
      if (beta) s2 += (double)beta[k] * orig;
    }
    if (layer_norm) {
      (*c1)[n] = (float)s1;
      (*c2)[n] = (float)s2;
    }
  }
}

template <typename T>
inline int RepackTyped(const ShahdModelCfg& c, const ParamLayout& lay, const T* p, HostWeights* hw) {
  const int E = c.embed_dim, H = c.num_heads, Hk = c.kv_heads, d = E / H, F = c.mlp_hidden, V = c.vocab_size;
  const int C = c.block_size;
  const int Ep = RoundUp(E, 8), Fp = RoundUp(F, 8), HDp = RoundUp(H * d, 8);
  for (int64_t i = 0; i < lay.total; i++)
    if (!std::isfinite((double)p[i])) {
      SetError("shahd_session_create: parameter %lld is not finite", (long long)i);
      return SHAHD_EINVAL;
    }
  auto bf = [](double v) { return __float2bfloat16_rn((float)v); };
  auto vec = [&](int64_t off, int64_t n) {
    std::vector<float> v(n);
    for (int64_t i = 0; i < n; i++) v[i] = (float)p[off + i];
    return v;
  };
  hw->layers.resize(c.num_layers);
  for (int l = 0; l < c.num_layers; l++) {
    const LayerParamOff& L = lay.layers[l];
    HostLayer& h = hw->layers[l];
    const int nqkv = (H + 2 * Hk) * d;
    const bool lnorm = c.norm_kind == 0;
    std::vector<float> g1 = vec(L.ln1_g, E), b1 = lnorm ? vec(L.ln1_b, E) : std::vector<float>();
    std::vector<float> g2 = vec(L.ln2_g, E), b2 = lnorm ? vec(L.ln2_b, E) : std::vector<float>();
    std::vector<float> wf((size_t)nqkv * E);
    for (int hh = 0; hh < H; hh++)
      for (int e = 0; e < E; e++)
        for (int j = 0; j < d; j++) wf[(size_t)(hh * d + j) * E + e] = (float)p[L.wq + (int64_t)hh * E * d + (int64_t)e * d + j];
    for (int g = 0; g < Hk; g++)
      for (int e = 0; e < E; e++)
        for (int j = 0; j < d; j++) {
          wf[(size_t)(H * d + g * d + j) * E + e] = (float)p[L.wk + (int64_t)g * E * d + (int64_t)e * d + j];
          wf[(size_t)((H + Hk) * d + g * d + j) * E + e] = (float)p[L.wv + (int64_t)g * E * d + (int64_t)e * d + j];
        }
    FoldNorm(wf, nqkv, E, Ep, g1.data(), lnorm ? b1.data() : nullptr, lnorm, &h.w_qkv, &h.qkv_c1, &h.qkv_c2);
    h.w_o.assign((size_t)E * HDp, bf(0));
    for (int hh = 0; hh < H; hh++)
      for (int j = 0; j < d; j++)
        for (int e = 0; e < E; e++)
          h.w_o[(size_t)e * HDp + hh * d + j] = bf(p[L.wo + (int64_t)hh * d * E + (int64_t)j * E + e]);
    if (c.mlp_kind == 0) {
      std::vector<float> uf((size_t)F * E);
      for (int e = 0; e < E; e++)
        for (int f = 0; f < F; f++) uf[(size_t)f * E + e] = (float)p[L.wfc + (int64_t)e * F + f];
      FoldNorm(uf, F, E, Ep, g2.data(), lnorm ? b2.data() : nullptr, lnorm, &h.w_up, &h.up_c1, &h.up_c2);
      h.b_fc = vec(L.bfc, F);
      h.w_down.assign((size_t)E * Fp, bf(0));
      for (int f = 0; f < F; f++)
        for (int e = 0; e < E; e++) h.w_down[(size_t)e * Fp + f] = bf(p[L.wproj + (int64_t)f * E + e]);
      h.b_proj = vec(L.bproj, E);
    } else {
      std::vector<float> uf((size_t)2 * F * E);
      for (int e = 0; e < E; e++)
        for (int f = 0; f < F; f++) {
          uf[(size_t)(2 * f) * E + e] = (float)p[L.w1 + (int64_t)e * F + f];
          uf[(size_t)(2 * f + 1) * E + e] = (float)p[L.w3 + (int64_t)e * F + f];
        }
      FoldNorm(uf, 2 * F, E, Ep, g2.data(), lnorm ? b2.data() : nullptr, lnorm, &h.w_up, &h.up_c1, &h.up_c2);
      h.w_down.assign((size_t)E * Fp, bf(0));
      for (int f = 0; f < F; f++)
        for (int e = 0; e < E; e++) h.w_down[(size_t)e * Fp + f] = bf(p[L.w2 + (int64_t)f * E + e]);
    }
  }
  {
    const bool lnorm = c.norm_kind == 0;
    std::vector<float> gf = vec(lay.lnf_g, E), bfv = lnorm ? vec(lay.lnf_b, E) : std::vector<float>();
    std::vector<float> hf((size_t)V * E);
    if (c.weight_tying) {
      for (int v = 0; v < V; v++)
        for (int e = 0; e < E; e++) hf[(size_t)v * E + e] = (float)p[lay.wte + (int64_t)v * E + e];
    } else {
      for (int e = 0; e < E; e++)
        for (int v = 0; v < V; v++) hf[(size_t)v * E + e] = (float)p[lay.lm_head + (int64_t)e * V + v];
    }
    FoldNorm(hf, V, E, Ep, gf.data(), lnorm ? bfv.data() : nullptr, lnorm, &hw->w_head, &hw->head_c1, &hw->head_c2);
  }
  hw->head_bias = vec(lay.lm_bias, V);
  hw->wte = vec(lay.wte, (int64_t)V * E);
  if (lay.wpe >= 0) hw->wpe = vec(lay.wpe, (int64_t)C * E);
  if (c.position_scheme == 1) {
    // RopeFrequencies / RopeCosSin (RotaryEmbedding.ts:17-38), computed in f64, stored fp32 [C, d/2].
    const double base = c.rope_base > 0 ? c.rope_base : 10000.0;
    const int half = d / 2;
    hw->rope_cos.resize((size_t)C * half);
    hw->rope_sin.resize((size_t)C * half);
    for (int i = 0; i < half; i++) {
      const double freq = std::pow(base, (-2.0 * i) / d);
      for (int pos = 0; pos < C; pos++) {
        const double ang = pos * freq;
        hw->rope_cos[(size_t)pos * half + i] = (float)std::cos(ang);
        hw->rope_sin[(size_t)pos * half + i] = (float)std::sin(ang);
      }
    }
  }
  (void)HDp;
  return SHAHD_OK;
}

inline int RepackWeights(const ShahdModelCfg& c, const ParamLayout& lay, const void* params, bool f64, HostWeights* hw) {
  return f64 ? RepackTyped(c, lay, static_cast<const double*>(params), hw)
             : RepackTyped(c, lay, static_cast<const float*>(params), hw);
}

// ---- the reference's weight initialization ---------------------------------------------------------

struct SeededRng {  // Brain/Random/SeededRng.ts:14-48
  uint32_t state;
  uint32_t NextU32() { return state = state * 1664525u + 1013904223u; }
  double NextFloat() { return (double)NextU32() / 4294967296.0; }
  double NextGaussian() {
    const double u = NextFloat(), v = NextFloat();
    return std::sqrt(-2.0 * std::log(u + 1e-12)) * std::cos(2.0 * M_PI * v);
  }
};

inline uint32_t MixSeed(uint32_t seed, uint32_t stream) {  // SeededRng.ts:7-12
  uint32_t x = seed ^ (uint32_t)((stream + 1u) * 0x9e3779b9u);
  x = (x ^ (x >> 16)) * 0x45d9f3bu;
  x = (x ^ (x >> 16)) * 0x45d9f3bu;
  return x ^ (x >> 16);
}

}  // namespace shahd

extern "C" int shahd_init_params(const ShahdModelCfg* cfg, uint32_t seed, float* params, int64_t count) {
  using namespace shahd;
  ClearError();
  ParamLayout lay;
  if (!cfg || !params || BuildParamLayout(*cfg, &lay) != SHAHD_OK) {
    if (!cfg || !params) SetError("shahd_init_params: null argument");
    return SHAHD_EINVAL;
  }
  if (count != lay.total) {
    SetError("shahd_init_params: count %lld != %lld", (long long)count, (long long)lay.total);
    return SHAHD_EINVAL;
  }
  const int64_t E = cfg->embed_dim, H = cfg->num_heads, Hk = cfg->kv_heads, d = E / H, F = cfg->mlp_hidden;
  const double s0 = 0.02, sres = 0.02 / std::sqrt(2.0 * cfg->num_layers);  // InitScale, ResidualInitScale
  SeededRng rng{MixSeed(seed, 0)};                                          // CreateRngStreams(seed).InitRng
  for (int64_t i = 0; i < count; i++) params[i] = 0.f;
  auto randn = [&](int64_t off, int64_t n, double scale) {
    for (int64_t i = 0; i < n; i++) params[off + i] = (float)(rng.NextGaussian() * scale);
  };
  auto fill1 = [&](int64_t off, int64_t n) {
    for (int64_t i = 0; i < n; i++) params[off + i] = 1.f;
  };
  randn(lay.wte, (int64_t)cfg->vocab_size * E, s0);
  if (lay.wpe >= 0) randn(lay.wpe, (int64_t)cfg->block_size * E, s0);
  for (int l = 0; l < cfg->num_layers; l++) {
    const LayerParamOff& L = lay.layers[l];
    fill1(L.ln1_g, E);
    for (int64_t h = 0; h < H; h++) {
      randn(L.wq + h * E * d, E * d, s0);
      randn(L.wo + h * d * E, d * E, sres);
    }
    for (int64_t g = 0; g < Hk; g++) {
      randn(L.wk + g * E * d, E * d, s0);
      randn(L.wv + g * E * d, E * d, s0);
    }
    fill1(L.ln2_g, E);
    if (cfg->mlp_kind == 0) {
      randn(L.wfc, E * F, s0);
      randn(L.wproj, F * E, sres);
    } else {
      randn(L.w1, E * F, s0);
      randn(L.w3, E * F, s0);
      randn(L.w2, F * E, sres);
    }
  }
  fill1(lay.lnf_g, E);
  if (lay.lm_head >= 0) randn(lay.lm_head, E * cfg->vocab_size, s0);
  return SHAHD_OK;
}
