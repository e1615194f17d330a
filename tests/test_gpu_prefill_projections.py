"""Batched-prefill projections on the persistent warp-specialized tcgen05 kernel against the oracle and
against the one-tile-per-CTA kernel they replace.

A prefill of many rows (ForwardHidden over the prompt, CachedForward.ts:100-110) runs every projection of
every layer over more than 128 rows: QKV with RoPE and the KV append, the summed O projection, the MLP up
projection with its activation and the down projection, each with its residual. The K/V rows the prefill
leaves in the cache for the deeper layers depend on all of them, so the logits of the decode steps that
follow check the whole prefill. Both norms (the persistent kernel takes the row statistics from a separate
pass over the fp32 residual), both MLP forms, learned positions and RoPE, tile edges in rows (ragged
prompts) and in columns (a vocabulary and MLP width that are not multiples of the 128/256-column tiles).
"""
import contextlib

import numpy as np
import pytest

from tests.helpers import O, TOL_BF16, greedy_agrees, oracle_shape, pkg, range_rel_err

pytestmark = pytest.mark.gpu

MODELS = [
    ("E256 RoPE RmsNorm SwiGlu GQA", dict(embed_dim=256, num_heads=4, kv_heads=2, position_scheme="Rope",
                                          norm_kind="RmsNorm", mlp_kind="SwiGlu", mlp_hidden=1024)),
    ("E128 learned LayerNorm Relu", dict(embed_dim=128, num_heads=4, mlp_hidden=520)),
    ("E192 RoPE LayerNorm GeGlu", dict(embed_dim=192, num_heads=3, position_scheme="Rope", mlp_kind="GeGlu",
                                       mlp_hidden=384)),
]


@contextlib.contextmanager
def persistent(enable: bool):
    lib = pkg.load()
    lib.ShahdSetPersistentPrefillProjections(1 if enable else 0)
    try:
        yield
    finally:
        lib.ShahdSetPersistentPrefillProjections(1)


def _steps(cfg, params, prompts, steps):
    n = len(prompts)
    with pkg.Session(cfg, params, max_seqs=n) as sess:
        sess.prefill(list(range(n)), [pr[:-1] for pr in prompts])
        toks = [int(pr[-1]) for pr in prompts]
        out = []
        for _ in range(steps):
            logits, nxt = sess.step(list(range(n)), toks)
            out.append((logits.copy(), nxt.copy()))
            toks = [int(t) for t in nxt]
    return out


@pytest.mark.parametrize("label,arch", MODELS, ids=[m[0] for m in MODELS])
def test_persistent_prefill_matches_oracle_and_tile_kernel(label, arch):
    cfg = pkg.ModelConfig(num_layers=2, block_size=256, vocab_size=1000, **arch)
    params = pkg.init_params(cfg, 29)
    model = O.Model(oracle_shape(cfg, "F32"), params.astype(np.float64))
    # 5 sequences, 431 prefill rows in one chunk (not a multiple of 128)
    prompts = [O.uniform_ids(n, cfg.vocab_size, seed=40 + i) for i, n in enumerate((150, 97, 64, 3, 122))]
    steps = 3
    with persistent(True):
        got = _steps(cfg, params, prompts, steps)
    with persistent(False):
        ref = _steps(cfg, params, prompts, steps)
    decs = [O.Decoder(model, pr) for pr in prompts]
    worst = worst_tile = 0.0
    same = True
    for k in range(steps):
        logits, nxt = got[k]
        for i in range(len(prompts)):
            want = decs[i].logits
            worst = max(worst, range_rel_err(logits[i], want))
            if same:
                worst_tile = max(worst_tile, range_rel_err(ref[k][0][i], want))
            assert greedy_agrees(nxt[i], want), (label, k, i)
            decs[i].push(int(nxt[i]))
        same = same and np.array_equal(nxt, ref[k][1])
    assert worst < TOL_BF16, (label, worst)
    assert worst_tile < TOL_BF16, (label, worst_tile)
    assert pkg.load().ShahdDeviceErrorFlag() == 0
