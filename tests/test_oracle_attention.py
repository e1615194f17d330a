"""The oracle's FusedAttention restatement (MultiHeadAttention.ts:46-74 core: RoPE, CausalSoftmax, @ V, GQA)
pinned on CPU: against a direct numpy restatement of the same formulas, the reference's relations
(fused vs unfused attention, FusedAttention.Test.ts:53-113; a row of the causal attention equals a decode
step's AttendRow over the rows before it, CachedRowMath.ts:60-86; RoPE keeps each pair's norm,
Phase2Ops.Test.ts:40-44) and a committed golden vector."""
import os

import numpy as np

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "oracle_golden.npz")


def _rope(x: np.ndarray, base: float) -> np.ndarray:
    T, _, d = x.shape
    x = x.copy()
    for t in range(T):
        for i in range(d // 2):
            a = t * base ** (-2.0 * i / d)
            c, s = np.cos(a), np.sin(a)
            x0, x1 = x[t, :, 2 * i].copy(), x[t, :, 2 * i + 1].copy()
            x[t, :, 2 * i] = x0 * c - x1 * s
            x[t, :, 2 * i + 1] = x0 * s + x1 * c
    return x


def _unfused(q, k, v, base):
    """Scale -> CausalMask -> SoftmaxRows, the chain CausalSoftmax replaces (CausalSoftmax.ts:1-11)."""
    T, H, d = q.shape
    G = H // k.shape[1]
    qr, kr = (_rope(q, base), _rope(k, base)) if base > 0 else (q, k)
    out = np.zeros_like(q)
    for h in range(H):
        s = (qr[:, h] @ kr[:, h // G].T) / np.sqrt(d)
        s = np.where(np.tril(np.ones((T, T))) > 0, s, -1e9)
        p = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h] = (p / p.sum(axis=1, keepdims=True)) @ v[:, h // G]
    return out


def test_fused_equals_unfused_chain():
    rng = np.random.default_rng(3)
    for T, H, Hk, d, base in ((1, 2, 1, 4, 10000.0), (9, 4, 2, 8, 10000.0), (33, 8, 2, 16, 500.0), (7, 3, 3, 6, 0.0)):
        q = rng.standard_normal((T, H, d))
        k = rng.standard_normal((T, Hk, d))
        v = rng.standard_normal((T, Hk, d))
        assert np.abs(O.fused_attention(q, k, v, base) - _unfused(q, k, v, base)).max() < 1e-12


def test_row_p_is_the_decode_step_over_rows_0_to_p():
    rng = np.random.default_rng(4)
    T, H, Hk, d = 20, 8, 2, 8
    q, k, v = rng.standard_normal((T, H, d)), rng.standard_normal((T, Hk, d)), rng.standard_normal((T, Hk, d))
    full = O.fused_attention(q, k, v)
    for p in (0, 1, 7, 19):
        prefix = O.fused_attention(q[: p + 1], k[: p + 1], v[: p + 1])
        assert np.abs(prefix[p] - full[p]).max() < 1e-12


def test_rope_keeps_pair_norms():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((16, 3, 10))
    r = _rope(x, 10000.0)
    assert np.allclose(x[..., 0::2] ** 2 + x[..., 1::2] ** 2, r[..., 0::2] ** 2 + r[..., 1::2] ** 2, atol=1e-12)


def test_fused_attention_golden_vector():
    g = np.load(GOLDEN)
    out = O.fused_attention(g["fa_q"], g["fa_k"], g["fa_v"], float(g["fa_base"]))
    assert np.array_equal(out, g["fa_out"])
