"""The fused decode attention block (one launch per layer: norm + Q/K/V projection + RoPE + KV append +
attention + output projection + residual, CachedForward.ts:66-84) against the oracle and against the
three-launch chain it replaces.

The block runs for decode rows whose rows x kv heads fill the SMs, on models whose Q/K/V rows of one kv
head fit in shared memory twice per SM. The cases cover both norms (the LayerNorm folding constants enter
the block's epilogue), learned positions and RoPE, one, two and four query heads per kv head, head_dim 32
and 64, an embedding width that leaves some lanes without a residual chunk (E = 192), kv-head clusters of
2, 3 and 4 CTAs, and ragged prompts whose new positions straddle the 32-position task and 64-position page
boundaries. Every row's teacher-forced logits are compared with the oracle at every step
(CachedForwardStep, CachedForward.ts:94-96) and greedy ids must agree wherever the oracle's top-2 margin
exceeds the tolerance. The cases run in an order that shrinks and then grows the block's shared memory
(kernel attributes are per device and must follow the largest request).
"""
import contextlib

import numpy as np
import pytest

from tests.helpers import O, TOL_BF16, greedy_agrees, oracle_shape, pkg, range_rel_err

pytestmark = pytest.mark.gpu

CASES = [
    # label, model, rows (rows x kv heads >= 148 SMs: one CTA per (row, kv head))
    ("MicroChat layer: E256 d64 G1, RoPE RmsNorm SwiGlu", dict(embed_dim=256, num_heads=4, position_scheme="Rope",
                                                                 norm_kind="RmsNorm", mlp_kind="SwiGlu"), 64),
    ("E128 d32 G2, learned LayerNorm Relu", dict(embed_dim=128, num_heads=4, kv_heads=2), 80),
    ("E256 d32 G4, RoPE LayerNorm GeGlu", dict(embed_dim=256, num_heads=8, kv_heads=2, position_scheme="Rope",
                                               mlp_kind="GeGlu"), 80),
    ("E192 d64 G1, RoPE RmsNorm (partial lanes)", dict(embed_dim=192, num_heads=3, position_scheme="Rope",
                                                       norm_kind="RmsNorm", mlp_kind="SwiGlu"), 64),
]


@contextlib.contextmanager
def fused_block(enable: bool):
    lib = pkg.load()
    lib.ShahdSetFusedAttentionBlock(1 if enable else 0)
    try:
        yield
    finally:
        lib.ShahdSetFusedAttentionBlock(0)


def _run(cfg, params, rows, prompts, steps, fused):
    with fused_block(fused), pkg.Session(cfg, params, max_seqs=rows) as sess:
        sess.prefill(list(range(rows)), [pr[:-1] for pr in prompts])
        launches = sess.step_launches(rows)
        toks = [int(pr[-1]) for pr in prompts]
        out = []
        for _ in range(steps):
            logits, nxt = sess.step(list(range(rows)), toks)
            out.append((logits.copy(), nxt.copy()))
            toks = [int(t) for t in nxt]
    return out, launches


@pytest.mark.parametrize("label,arch,rows", CASES, ids=[c[0] for c in CASES])
def test_fused_block_matches_oracle_and_chain(label, arch, rows):
    cfg = pkg.ModelConfig(num_layers=2, block_size=160, vocab_size=512, mlp_hidden=2 * arch["embed_dim"], **arch)
    params = pkg.init_params(cfg, 17)
    model = O.Model(oracle_shape(cfg, "F32"), params.astype(np.float64))
    # new positions from 29 to 96 over the steps: crossing positions 31/32 (task) and 63/64 (page)
    prompts = [O.uniform_ids(30 + (11 * i) % 64, cfg.vocab_size, seed=300 + i) for i in range(rows)]
    steps = 4
    fused, n_fused = _run(cfg, params, rows, prompts, steps, True)
    chain, n_chain = _run(cfg, params, rows, prompts, steps, False)
    assert n_fused == 1 + 3 * cfg.num_layers + 2, "the fused block was not selected for this shape"
    assert n_chain == 1 + 5 * cfg.num_layers + 2
    decs = [O.Decoder(model, pr) for pr in prompts]
    worst = worst_chain = 0.0
    same = True  # the chain is fed its own ids: its logits are comparable while both trajectories agree
    for k in range(steps):
        logits, nxt = fused[k]
        for i in range(rows):
            want = decs[i].logits
            worst = max(worst, range_rel_err(logits[i], want))
            if same:
                worst_chain = max(worst_chain, range_rel_err(chain[k][0][i], want))
            assert greedy_agrees(nxt[i], want), (label, k, i)
            decs[i].push(int(nxt[i]))
        same = same and np.array_equal(nxt, chain[k][1])
    assert worst < TOL_BF16, (label, worst)
    assert worst_chain < TOL_BF16, (label, worst_chain)
    assert pkg.load().ShahdDeviceErrorFlag() == 0


def test_fused_block_generate_is_deterministic_and_matches_oracle():
    # the decode loop of CachedGenerate over the fused block, past the 384-position mean length at which the
    # three-launch chain switches to the page-streaming attention kernel
    cfg = pkg.ModelConfig(embed_dim=256, num_layers=2, num_heads=4, block_size=512, vocab_size=512,
                          mlp_hidden=512, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")
    params = pkg.init_params(cfg, 23)
    model = O.Model(oracle_shape(cfg, "F32"), params.astype(np.float64))
    rows = 64
    prompts = np.stack([O.uniform_ids(380, cfg.vocab_size, seed=700 + i) for i in range(rows)])
    with fused_block(True), pkg.Session(cfg, params, max_seqs=rows) as sess:
        assert sess.step_launches(rows) == 1 + 3 * cfg.num_layers + 2
        ids = sess.generate(prompts, 40)
        again = sess.generate(prompts, 40)
    assert np.array_equal(ids, again), "the fused block is not deterministic run to run"
    chk = model.check_trajectories(prompts, ids, TOL_BF16)
    assert int(chk["fails"].sum()) == 0, np.nonzero(chk["fails"])[0][:8]
    assert pkg.load().ShahdDeviceErrorFlag() == 0
