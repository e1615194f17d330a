"""Greedy speculative decoding (SpeculativeDecodeGreedy, Brain/Reasoning/SpeculativeDecode.ts:32-98) on GPU
sessions: within the window the ids are plain greedy decoding with the target (SpeculativeDecode.ts:5-10),
whatever the draft; a draft identical to the target has its proposals accepted. The verify pass and the
per-step path round differently, so an id may only differ where the oracle's top-2 margin is within
tolerance."""
import numpy as np
import pytest

from tests.helpers import O, TOL_BF16, oracle_shape, pkg

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
