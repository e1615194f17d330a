"""The decode workloads this backend is measured and checked on (shapes of the reference's configs).

Each entry: the model shape (mapped onto the reference's Model knobs, Brain/Config/ValidateConfig.ts:32-49),
the weight seed, and the decode job (independent sequences, uniform prompt ids, greedy new tokens).
"""
from __future__ import annotations

from dataclasses import dataclass

from .decode import ModelConfig


@dataclass(frozen=True)
class Workload:
    name: str
    model: ModelConfig
    weight_seed: int
    seqs: int
    prompt_len: int
    new_tokens: int


# emb 128, 4 layers, 4 heads (d 32), learned positions, ctx 256, vocab 4096, tied. "MLP 4x GELU" maps to
# the reference's only GELU MLP, the gated GeGlu (Brain/Nn/Mlp.ts:2-4), hidden 512; LayerNorm (default).
FOUNDRY = Workload(
    "foundry-shape E128 L4 H4 GeGlu F512 ctx256 V4096",
    ModelConfig(embed_dim=128, num_layers=4, num_heads=4, block_size=256, vocab_size=4096, mlp_hidden=512,
                position_scheme="Learned", norm_kind="LayerNorm", mlp_kind="GeGlu"),
    weight_seed=0, seqs=1, prompt_len=64, new_tokens=192)

# emb 256, 6 layers, 4 heads (d 64), MLP 4x (F 1024), ctx 512, vocab 4096, tied; MicroChat training recipe:
# Rope + RmsNorm + SwiGlu (Scripts/TrainOnFoundry.ts:232).
MICROCHAT = Workload(
    "MicroChat-shape E256 L6 H4 SwiGlu F1024 ctx512 V4096",
    ModelConfig(embed_dim=256, num_layers=6, num_heads=4, block_size=512, vocab_size=4096, mlp_hidden=1024,
                position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu"),
    weight_seed=1, seqs=64, prompt_len=128, new_tokens=384)

# emb 1024, 16 layers, 16 query / 4 KV heads (d 64), RmsNorm, Rope, SwiGlu 2816, ctx 2048, vocab 32768, tied.
PHASE2 = Workload(
    "Phase2Modern-style E1024 L16 H16/4 SwiGlu F2816 ctx2048 V32768",
    ModelConfig(embed_dim=1024, num_layers=16, num_heads=16, kv_heads=4, block_size=2048, vocab_size=32768,
                mlp_hidden=2816, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu"),
    weight_seed=4, seqs=4096, prompt_len=512, new_tokens=512)

WORKLOADS = {"foundry": FOUNDRY, "microchat": MICROCHAT, "phase2": PHASE2}
