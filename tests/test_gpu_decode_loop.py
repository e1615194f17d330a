"""The persistent cluster decode loop (greedy generate) against the oracle, logits and ids, over the shapes
its fixed work split admits: head_dim 32 and 64, 1-4 query heads per kv head, RoPE and learned positions,
RmsNorm and LayerNorm, SwiGLU / GeGLU / ReLU MLPs, tied and untied heads, vocabularies that are not a
multiple of the 128-row tile, 1 to 40 rows (one or several clusters, full and partial row groups), and runs
that cross the context window (the loop stops, the cache is rebuilt from the last BlockSize-1 ids,
CachedForward.ts:133-141, and the loop resumes).

Each run records every step's logits (shahd_generate_logits); the oracle's CachedDecoder, pushed the GPU's
own ids, must agree within 2e-2 of the logit range at every step (CachedForward.Test.ts:46-55 relation on
the decode loop), and every id must be the oracle's argmax outside near ties.
"""
import numpy as np
import pytest

from tests.helpers import O, TOL_BF16, decode_loop, greedy_agrees, oracle_shape, pkg, range_rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _loop_on():
    with decode_loop(True):  # an opt-in path: every test of this file runs greedy generate through it
        yield

LOOP_ARCHS = [
    ("E256 d64 GQA4/2 SwiGLU RmsNorm RoPE",
     dict(embed_dim=256, num_layers=2, num_heads=4, kv_heads=2, block_size=256, vocab_size=1024, mlp_hidden=512,
          position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")),
    ("E256 d32 GQA8/2 ReLU LayerNorm learned V1000",
     dict(embed_dim=256, num_layers=2, num_heads=8, kv_heads=2, block_size=256, vocab_size=1000, mlp_hidden=512,
          position_scheme="Learned", norm_kind="LayerNorm", mlp_kind="Relu")),
    ("foundry-like E128 d32 GeGLU LayerNorm learned",
     dict(embed_dim=128, num_layers=2, num_heads=4, block_size=256, vocab_size=4096, mlp_hidden=512,
          position_scheme="Learned", norm_kind="LayerNorm", mlp_kind="GeGlu")),
    ("E512 d64 Hk8 untied SwiGLU RoPE V777",
     dict(embed_dim=512, num_layers=1, num_heads=8, kv_heads=8, block_size=256, vocab_size=777, mlp_hidden=1024,
          position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu", weight_tying=False)),
]


def _check_run(cfg, params, prompts, new, rows_checked=None):
    model = O.Model(oracle_shape(cfg, "F32"), params.astype(np.float64))
    with pkg.Session(cfg, params, max_seqs=len(prompts)) as sess:
        ids, logits = sess.generate_logits(prompts, new)
        plain = sess.generate(prompts, new)
    assert np.array_equal(ids, plain), "logits recording changed the ids"
    worst = 0.0
    for i in (rows_checked if rows_checked is not None else range(len(prompts))):
        dec = O.Decoder(model, prompts[i])
        for k in range(new):
            want = dec.logits
            worst = max(worst, range_rel_err(logits[i, k], want))
            assert greedy_agrees(ids[i, k], want), (i, k)
            if k + 1 < new:
                dec.push(int(ids[i, k]))
    assert worst < TOL_BF16, worst
    assert pkg.load().ShahdDeviceErrorFlag() == 0
    return ids


@pytest.mark.parametrize("label,arch", LOOP_ARCHS, ids=[a[0] for a in LOOP_ARCHS])
@pytest.mark.parametrize("nrows", [1, 5, 40])
def test_decode_loop_logits_match_oracle(label, arch, nrows):
    cfg = pkg.ModelConfig(**arch)
    params = pkg.init_params(cfg, 7)
    prompts = [O.uniform_ids(20 + (13 * i) % 90, cfg.vocab_size, seed=800 + i) for i in range(nrows)]
    checked = range(nrows) if nrows <= 5 else [0, 1, 17, 39]
    _check_run(cfg, params, prompts, 12, checked)


def test_decode_loop_crosses_the_window():
    # block 64, prompts of 50-60 ids, 40 new ids: every row slides its window at least once mid-run
    cfg = pkg.ModelConfig(embed_dim=256, num_layers=2, num_heads=4, kv_heads=4, block_size=64, vocab_size=512,
                          mlp_hidden=512, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")
    params = pkg.init_params(cfg, 3)
    prompts = [O.uniform_ids(50 + i, cfg.vocab_size, seed=60 + i) for i in range(11)]
    _check_run(cfg, params, prompts, 40)


def test_decode_loop_state_continues_into_cached_steps():
    # after a loop run the cache, the lengths and the next input are the host's view: a cached step on the
    # same slot continues the sequence exactly like the oracle's decoder
    w = pkg.configs.MICROCHAT
    cfg = w.model
    params = pkg.init_params(cfg, w.weight_seed)
    model = O.Model(oracle_shape(cfg, "F32"), params.astype(np.float64))
    prompts = [O.uniform_ids(30, cfg.vocab_size, seed=90 + i) for i in range(3)]
    with pkg.Session(cfg, params, max_seqs=3) as sess:
        ids = sess.generate(prompts, 10)
        for i in range(3):
            # generate leaves prompt (30) + 9 pushed ids in the cache; the 10th id is the next input
            assert sess.length(i) == 30 + 9
        logits, nxt = sess.step([0, 1, 2], [int(ids[i, -1]) for i in range(3)])
    for i in range(3):
        dec = O.Decoder(model, prompts[i])
        for t in ids[i]:
            dec.push(int(t))
        assert range_rel_err(logits[i], dec.logits) < TOL_BF16
        assert greedy_agrees(nxt[i], dec.logits)
