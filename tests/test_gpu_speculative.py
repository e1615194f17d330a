"""Greedy speculative decoding (SpeculativeDecodeGreedy, Brain/Reasoning/SpeculativeDecode.ts:32-98) on GPU
sessions: within the window the ids are plain greedy decoding with the target (SpeculativeDecode.ts:5-10),
whatever the draft; a draft identical to the target has its proposals accepted. The verify pass and the
per-step path round differently, so an id may only differ where the oracle's top-2 margin is within
tolerance."""
import numpy as np
import pytest

from tests.helpers import O, TOL_BF16, oracle_shape, pkg, range_rel_err

pytestmark = pytest.mark.gpu


def _near_tie_ok(model, prompt, a, b):
    """First index where a and b differ must be a near tie of the oracle (teacher-forced on a)."""
    if a == b:
        return True
    k = next(j for j in range(min(len(a), len(b))) if a[j] != b[j])
    odec = O.Decoder(model, prompt)
    for t in a[:k]:
        odec.push(int(t))
    s = np.sort(odec.logits)
    return s[-1] - s[-2] <= TOL_BF16 * (odec.logits.max() - odec.logits.min())


def _setup(n=4, plen=32):
    w = pkg.configs.MICROCHAT
    cfg = w.model
    p = pkg.init_params(cfg, w.weight_seed)
    prompts = [O.uniform_ids(plen, cfg.vocab_size, seed=600 + i).tolist() for i in range(n)]
    return cfg, p, prompts


@pytest.mark.parametrize("draft_kind", ["same", "other"])
def test_speculative_equals_plain_greedy(draft_kind):
    cfg, p, prompts = _setup()
    new, gamma = 40, 4
    if draft_kind == "same":
        dcfg, dp = cfg, p
    else:  # a smaller, differently seeded draft
        dcfg = pkg.ModelConfig(**{**cfg.__dict__, "num_layers": 2})
        dp = pkg.init_params(dcfg, 77)
    with pkg.Session(cfg, p, max_seqs=4) as tgt, pkg.Session(dcfg, dp, max_seqs=4) as drf:
        plain = tgt.generate(np.array(prompts), new)
        res = pkg.speculative.speculative_decode_greedy(tgt, drf, prompts, new, gamma)
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    for i, pr in enumerate(prompts):
        spec = res.ids[i][len(pr):]
        assert len(spec) == new
        assert _near_tie_ok(model, pr, plain[i].tolist(), spec), i
        assert res.draft_tokens[i] >= res.accepted_tokens[i]
    if draft_kind == "same":
        assert sum(res.accepted_tokens) >= 0.9 * sum(res.draft_tokens)
        assert max(res.target_calls) <= -(-new // (gamma + 1)) + 2
    assert pkg.load().ShahdDeviceErrorFlag() == 0


def test_verify_matches_steps_and_truncate_rewinds():
    cfg, p, prompts = _setup(n=2, plen=20)
    extra = [[5, 9, 2, 7], [1, 3]]
    with pkg.Session(cfg, p, max_seqs=2) as s:
        s.prefill([0, 1], prompts)
        got, lg = s.verify([0, 1], extra, want_logits=True)
        assert s.length(0) == 24 and s.length(1) == 22
        for i in range(2):
            assert np.array_equal(got[i], np.argmax(lg[i], axis=1))  # first index of the max
        s.truncate([0, 1], [20, 20])
        for j in range(2):  # stepping from the rewound length reproduces the verify rows
            step_lg, _ = s.step([0, 1], [extra[0][j], extra[1][j]])
            for i in range(2):
                rng = lg[i][j].max() - lg[i][j].min()
                assert np.abs(step_lg[i] - lg[i][j]).max() / rng < TOL_BF16
        with pytest.raises(pkg._lib.ShahdError, match="cannot keep"):
            s.truncate([0], [50])
        with pytest.raises(pkg._lib.ShahdError, match="window"):
            s.verify([0], [[1] * (cfg.block_size)])


# ---- stochastic speculative sampling (Brain/Reasoning/SpeculativeSampling.ts) -------------------------

def test_device_round_matches_the_oracle_on_given_logits():
    # one round per sequence on caller logits: accepted proposals, the residual / bonus id and the Rng state
    # must be the oracle's (SpeculativeSampling.ts:82-112 restated) exactly
    import ctypes

    rng = np.random.default_rng(12)
    lib = pkg.load()
    V, gamma, n = 300, 4, 48
    for temperature, top_k, top_p in ((1.0, 0, 1.0), (0.7, 40, 0.9), (1.3, 0, 0.8)):
        tl = (rng.standard_normal((n, gamma + 1, V)) * 2).astype(np.float32)
        dl = (tl[:, :gamma] + rng.standard_normal((n, gamma, V)).astype(np.float32) * 0.5).astype(np.float32)
        dl[:4] = tl[:4, :gamma]  # drafts equal to the target: every proposal accepted
        props = rng.integers(0, V, (n, gamma)).astype(np.int32)
        props[:8] = np.argmax(dl[:8], axis=2)  # likely proposals too
        g = rng.integers(0, gamma + 1, n).astype(np.int32)
        g[:4] = gamma
        budget = rng.integers(1, 8, n).astype(np.int32)
        budget[:4] = 10
        st = rng.integers(1, 2**32, n, dtype=np.uint64).astype(np.uint32)
        st0 = st.copy()
        out = np.zeros((n, gamma + 1), np.int32)
        cnt = np.zeros(n, np.int32)
        acc = np.zeros(n, np.int32)
        o = pkg.Sampling(temperature, top_k, top_p).to_c()
        fp, ip = ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int32)
        pkg._lib.check(lib.shahd_speculative_round(
            tl.ctypes.data_as(fp), dl.ctypes.data_as(fp), props.ctypes.data_as(ip), g.ctypes.data_as(ip),
            budget.ctypes.data_as(ip), n, gamma, V, ctypes.byref(o), st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
            out.ctypes.data_as(ip), cnt.ctypes.data_as(ip), acc.ctypes.data_as(ip)))
        for i in range(n):
            want, want_acc, want_st = O.speculative_round(tl[i, : g[i] + 1].astype(np.float64),
                                                          dl[i, : g[i]].astype(np.float64), props[i, : g[i]],
                                                          int(budget[i]), int(st0[i]), temperature, top_k, top_p)
            assert out[i, : cnt[i]].tolist() == want, (temperature, i)
            assert int(acc[i]) == want_acc and int(st[i]) == want_st, (temperature, i)
        assert all(int(acc[i]) == min(gamma, int(budget[i])) for i in range(4))  # q == p accepts everything


def test_speculative_sample_replays_with_the_oracle():
    # two GPU sessions (target, weaker draft); every decision of every round is replayed with the oracle on the
    # logits the GPU used: the draft's proposals (one draw each from its distribution) and the round's accept /
    # residual / bonus ids, with the Rng states carried through; the target's logits agree with the oracle's
    target_cfg = pkg.ModelConfig(embed_dim=64, num_layers=2, num_heads=4, block_size=64, vocab_size=96,
                                 mlp_hidden=128, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")
    draft_cfg = pkg.ModelConfig(embed_dim=64, num_layers=1, num_heads=4, block_size=64, vocab_size=96,
                                mlp_hidden=128, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")
    tp, dp = pkg.init_params(target_cfg, 7), pkg.init_params(draft_cfg, 11)
    tmodel = O.Model(oracle_shape(target_cfg, "F32"), tp.astype(np.float64))
    prompts = [[4, 5, 6], [1, 2, 3, 7, 8], [9]]
    samp = pkg.Sampling(1.0, 10, 0.95)
    rng_states = np.array([2, 3, 4], np.uint32)
    with pkg.Session(target_cfg, tp, max_seqs=3) as t, pkg.Session(draft_cfg, dp, max_seqs=3) as d:
        res, rounds = pkg.speculative.speculative_sample(t, d, prompts, 20, samp, rng_states, gamma=4, record=True)
    for p, ids in zip(prompts, res.ids):
        assert len(ids) == len(p) + 20 and all(0 <= x < 96 for x in ids)
    assert sum(res.accepted_tokens) <= sum(res.draft_tokens)
    state = {i: None for i in range(3)}
    for r in rounds:
        if state[r.seq] is not None:
            assert r.rng_at_start == state[r.seq]  # draws continue where the last round left them
        st = r.rng_at_start
        for k, tok in enumerate(r.proposals):
            want, st = O.sample_from_logits(r.draft_logits[k].astype(np.float64), st, 1.0, 10, 0.95)
            assert want == tok
        assert st == r.rng_before_round
        ids, acc, st = O.speculative_round(r.target_logits.astype(np.float64), r.draft_logits.astype(np.float64),
                                           r.proposals, r.budget, r.rng_before_round, 1.0, 10, 0.95)
        assert ids == r.appended and acc == r.accepted
        state[r.seq] = st
    assert [state[i] for i in range(3)] == rng_states.tolist()
    # the target rows of the first round of sequence 0 against the oracle's forward on the same ids
    r0 = next(r for r in rounds if r.seq == 0)
    ctx = prompts[0] + r0.proposals
    full = tmodel.forward(ctx)
    for k in range(len(r0.proposals) + 1):
        assert range_rel_err(r0.target_logits[k], full[len(prompts[0]) - 1 + k]) < TOL_BF16
