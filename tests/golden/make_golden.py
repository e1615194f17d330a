"""Generates tests/golden/oracle_golden.npz: pinned outputs of the CPU oracle and of the reference's
own C matmul kernels (oracle/_ref), so a later change to either shows up as a fixture mismatch.

    python -m tests.golden.make_golden        # from the repository root
"""
import ctypes
import os

import numpy as np

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))

# The BASELINE foundry-shape decoder (GeGlu stands in for "MLP 4x GELU": the reference's only GELU MLP
# is gated, Brain/Nn/Mlp.ts:2-4), reduced to 2 layers so the fixture builds in well under a second.
SMALL = O.Shape(embed_dim=128, num_layers=2, num_heads=4, block_size=32, vocab_size=512, mlp_hidden=512,
                mlp_kind="GeGlu", precision="F32")
MICRO = O.Shape(embed_dim=64, num_layers=2, num_heads=4, kv_heads=2, block_size=24, vocab_size=256, mlp_hidden=128,
                position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu", precision="F32")


def compute_goldens() -> dict:
    out = {}
    for name, shape, seed in (("small", SMALL, 0), ("micro", MICRO, 1)):
        p = O.init_params(shape, seed)
        out[f"{name}_params_head"] = p[:64].copy()
        out[f"{name}_params_sum"] = np.array([p.sum(), np.abs(p).sum()])
        model = O.Model(shape, p)
        prompt = O.uniform_ids(10, shape.vocab_size, seed=7)
        ids, _ = model.cached_generate(prompt, 30)  # runs past the window (block 24/32) for micro
        out[f"{name}_greedy_ids"] = ids
        cache = model.new_cache()
        logits = np.stack([cache.step(int(t)) for t in prompt[:6]])
        out[f"{name}_step_logits"] = logits
        sids, st = model.cached_generate(prompt, 12, temperature=0.8, top_k=20, top_p=0.9, rng_state=11)
        out[f"{name}_sampled_ids"] = np.append(sids, np.int32(st & 0x7FFFFFFF)).astype(np.int64)
    # FusedAttention restatement (RoPE base 10000, GQA 4/2, causal), Q/K/V N(0,1) seed 3
    rng = np.random.default_rng(3)
    out["fa_q"] = rng.standard_normal((12, 4, 8))
    out["fa_k"] = rng.standard_normal((12, 2, 8))
    out["fa_v"] = rng.standard_normal((12, 2, 8))
    out["fa_base"] = np.array(10000.0)
    out["fa_out"] = O.fused_attention(out["fa_q"], out["fa_k"], out["fa_v"], 10000.0)
    R = O.ref_lib()
    if R is not None:
        rng = np.random.default_rng(2)
        a = rng.standard_normal((33, 70)).astype(np.float32)
        bt = rng.standard_normal((19, 70)).astype(np.float32)
        c = np.empty((33, 19), dtype=np.float32)
        fp = ctypes.POINTER(ctypes.c_float)
        R.RefMatMulNTF32(a.ctypes.data_as(fp), bt.ctypes.data_as(fp), c.ctypes.data_as(fp), 33, 70, 19, 0, 4)
        out["ref_nt_f32_a"], out["ref_nt_f32_bt"], out["ref_nt_f32_out"] = a, bt, c
    return out


if __name__ == "__main__":
    g = compute_goldens()
    np.savez_compressed(os.path.join(HERE, "oracle_golden.npz"), **g)
    print("wrote", sorted(g))
