"""Shared test helpers: the package import, config conversion to the oracle, parity metrics."""
from __future__ import annotations

import contextlib
import importlib

import numpy as np

pkg = importlib.import_module("shahd-llm-stack_b200")

from oracle import oracle as O  # noqa: E402

# north_star tolerances: per-step logits within max-abs 2e-2 (BF16) / 1e-4 (TF32/FP32) of the logit range
TOL_BF16 = 2e-2
TOL_F32 = 1e-4


@contextlib.contextmanager
def decode_loop(enable: bool):
    """Greedy generate through the persistent cluster decode loop (True) or per-kernel step chains (False, the
    library default), restoring the default afterwards."""
    lib = pkg.load()
    lib.ShahdSetPersistentStep(1 if enable else 0)
    try:
        yield
    finally:
        lib.ShahdSetPersistentStep(0)


def oracle_shape(cfg, precision: str = "F32") -> O.Shape:
    return O.Shape(
        embed_dim=cfg.embed_dim, num_layers=cfg.num_layers, num_heads=cfg.num_heads, block_size=cfg.block_size,
        vocab_size=cfg.vocab_size, mlp_hidden=cfg.mlp_hidden, kv_heads=cfg.kv, position_scheme=cfg.position_scheme,
        norm_kind=cfg.norm_kind, mlp_kind=cfg.mlp_kind, weight_tying=cfg.weight_tying, precision=precision,
        layer_norm_eps=cfg.layer_norm_eps)


def range_rel_err(got: np.ndarray, want: np.ndarray) -> float:
    """max|got - want| / (max(want) - min(want)) — the north_star logits metric."""
    rng = float(np.max(want) - np.min(want))
    return float(np.max(np.abs(got.astype(np.float64) - want))) / max(rng, 1e-30)


def top2_margin(logits: np.ndarray) -> float:
    s = np.sort(np.asarray(logits, dtype=np.float64))
    return float(s[-1] - s[-2]) if s.size > 1 else float("inf")


def greedy_agrees(gpu_id: int, oracle_logits: np.ndarray, tol: float = TOL_BF16) -> bool:
    """Greedy ids must match wherever the oracle's top-2 margin exceeds tol x logit range."""
    rng = float(np.max(oracle_logits) - np.min(oracle_logits))
    if top2_margin(oracle_logits) <= tol * rng:
        return True
    return int(gpu_id) == O.argmax(oracle_logits)


# Tests/CachedForward.Test.ts:15-25 — the six architectures of the reference's relational tests
SHARED = dict(embed_dim=16, num_layers=2, block_size=8, vocab_size=12, mlp_hidden=32)
ARCHS = [
    ("Learned/LayerNorm/Relu/MHA", dict(SHARED, num_heads=2)),
    ("Learned/LayerNorm/Relu/MHA untied", dict(SHARED, num_heads=1, weight_tying=False)),
    ("Rope/RmsNorm/SwiGlu/MHA", dict(SHARED, num_heads=4, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")),
    ("Rope/RmsNorm/SwiGlu/GQA 2-of-4",
     dict(SHARED, num_heads=4, kv_heads=2, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")),
    ("Rope/LayerNorm/Relu", dict(SHARED, num_heads=2, position_scheme="Rope")),
    ("Learned/RmsNorm/GeGlu/GQA 1-of-2", dict(SHARED, num_heads=2, kv_heads=1, norm_kind="RmsNorm", mlp_kind="GeGlu")),
]
