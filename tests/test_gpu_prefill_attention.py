"""Causal prefill attention (MultiHeadAttention.ts:46-74 with CausalSoftmax.ts:17-33) against the oracle, on
both kernels that serve it: the tensor-core kernel (head_dim 64: tcgen05 Q.K^T and P.V tiles in TMEM over
TMA-streamed pages, 128-query blocks) and the CUDA-core tile kernel (64-query blocks, fp32 products).

A batched prefill writes every layer's K/V rows from the previous layer's attention output, so the cache the
first decode steps read depends on the prefill attention of every prompt row. Prompt lengths straddle the
64-position pages and the 128-query blocks (prefills of 1, 63, 64, 65, 127, 128, 129 ... 510 rows);
each row's logits over the next steps are compared with the oracle's CachedDecoder, and the two kernels'
logits with each other.
"""
import numpy as np
import pytest

from tests.helpers import O, TOL_BF16, greedy_agrees, oracle_shape, pkg, range_rel_err

pytestmark = pytest.mark.gpu

CASES = [
    ("d64 G4 Hk2 (FusedAttention heads)", dict(embed_dim=512, num_heads=8, kv_heads=2)),
    ("d64 G1 Hk4 (MicroChat heads)", dict(embed_dim=256, num_heads=4, kv_heads=4)),
    ("d64 G2 Hk4", dict(embed_dim=512, num_heads=8, kv_heads=4)),
]
LENGTHS = [2, 64, 65, 66, 128, 129, 130, 200, 257, 384, 450, 511]  # prompt lengths (prefill = length - 1)


@pytest.mark.parametrize("label,arch", CASES, ids=[c[0] for c in CASES])
def test_prefill_attention_kernels_match_oracle(label, arch):
    cfg = pkg.ModelConfig(num_layers=2, block_size=512, vocab_size=512, mlp_hidden=2 * arch["embed_dim"],
                          position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu", **arch)
    p = pkg.init_params(cfg, 21)
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    prompts = [O.uniform_ids(n, cfg.vocab_size, seed=1300 + i) for i, n in enumerate(LENGTHS)]
    rows = list(range(len(prompts)))
    lib = pkg.load()
    steps = 2
    got = {}
    for tc in (1, 0):
        lib.ShahdSetTensorCorePrefillAttention(tc)
        try:
            with pkg.Session(cfg, p, max_seqs=len(prompts)) as sess:
                sess.prefill(rows, [pr[:-1] for pr in prompts])
                toks = [int(pr[-1]) for pr in prompts]
                out = []
                for _ in range(steps):
                    logits, nxt = sess.step(rows, toks)
                    out.append((logits.copy(), nxt.copy()))
                    toks = [int(v) for v in nxt]
                got[tc] = out
        finally:
            lib.ShahdSetTensorCorePrefillAttention(1)
    assert lib.ShahdDeviceErrorFlag() == 0
    O.set_threads(8)
    try:
        decs = [O.Decoder(model, pr) for pr in prompts]
    finally:
        O.set_threads(1)
    worst = {0: 0.0, 1: 0.0}
    cross = 0.0
    diverged = set()  # rows whose CUDA-core run took another id at a near tie: compared only up to it
    for t in range(steps):
        for i in rows:
            want = decs[i].logits
            for tc in (1, 0):
                if tc == 0 and i in diverged:
                    continue
                lg, nxt = got[tc][t]
                worst[tc] = max(worst[tc], range_rel_err(lg[i], want))
                assert greedy_agrees(nxt[i], want), (label, tc, i, t)
            if i not in diverged:
                cross = max(cross, range_rel_err(got[1][t][0][i], got[0][t][0][i]))
                if got[0][t][1][i] != got[1][t][1][i]:
                    diverged.add(i)
        if t + 1 < steps:
            for i in rows:  # the oracle is teacher-forced on the tensor-core run's ids
                decs[i].push(int(got[1][t][1][i]))
    assert worst[1] < TOL_BF16, (label, worst)
    assert worst[0] < TOL_BF16, (label, worst)
    assert cross < TOL_BF16, (label, cross)


def test_long_prefill_of_many_sequences_fills_the_grid():
    # 40 sequences x 511 prefill rows in one batched prefill: several chunks, 4 query blocks per sequence,
    # more CTAs than are resident at once; four rows checked against the oracle
    cfg = pkg.ModelConfig(embed_dim=512, num_layers=1, num_heads=8, kv_heads=2, block_size=512, vocab_size=512,
                          mlp_hidden=1024, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")
    p = pkg.init_params(cfg, 5)
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    n = 40
    prompts = [O.uniform_ids(511 - (i % 3), cfg.vocab_size, seed=1500 + i) for i in range(n)]
    with pkg.Session(cfg, p, max_seqs=n) as sess:
        sess.prefill(list(range(n)), [pr[:-1] for pr in prompts])
        logits, nxt = sess.step(list(range(n)), [int(pr[-1]) for pr in prompts])
    assert pkg.load().ShahdDeviceErrorFlag() == 0
    O.set_threads(8)
    try:
        for i in (0, 13, 26, 39):
            want = O.Decoder(model, prompts[i]).logits
            assert range_rel_err(logits[i], want) < TOL_BF16, i
            assert greedy_agrees(nxt[i], want), i
    finally:
        O.set_threads(1)
