"""Seeded sampling on the GPU against the oracle's SampleFromLogits (Sampler.ts:16-27,
Distribution.ts:35-104).

The sampler itself is compared on logits both sides share exactly (quantized to 1/16 so that exact ties
occur and distinct values are far apart): RNG states must advance identically, and ids must be equal
unless a 1e-5 change of the draw or of TopP changes the oracle's own answer (the device keeps fp32
probabilities, the oracle f64). The decode loop is then checked by replaying its trajectory through
shahd_step and applying the oracle sampler to the step logits. Relations from
Tests/CachedForward.Test.ts:81-87 (same RNG, same ids) and the top-k/top-p order note of
Distribution.ts:61-64.
"""
import numpy as np
import pytest

from tests.helpers import ARCHS, O, pkg

pytestmark = pytest.mark.gpu

OPTS = [(1.0, 0, 1.0), (0.7, 40, 1.0), (1.3, 0, 0.9), (0.8, 50, 0.95), (1.0, 1, 1.0), (1.0, 0, 0.0),
        (1.0, 10 ** 6, 1.0), (0.5, 3, 0.5)]


def quantized_logits(seed, rows, vocab, scale):
    rng = np.random.default_rng(seed)
    return (np.round(rng.standard_normal((rows, vocab)) * scale * 16) / 16).astype(np.float32)


def explainable(logits, t, k, p, state_after, got):
    """True if the oracle picks `got` for a draw or TopP within 1e-5 of the exact ones."""
    u = state_after / 2.0 ** 32
    for dp in ((0.0, -1e-5, 1e-5) if p < 1 else (0.0,)):
        pp = p if p >= 1 else min(max(p + dp, 0.0), 1.0 - 1e-12)
        probs = O.probs_from_logits(np.asarray(logits, np.float64), t, k, pp)
        cum = np.cumsum(probs)
        nz = np.nonzero(probs > 0)[0]
        for du in (0.0, -1e-5, 1e-5):
            hit = nz[cum[nz] >= u + du]
            if (int(hit[0]) if hit.size else int(nz[-1])) == got:
                return True
    return False


def oracle_rows(logits, states, t, k, p):
    ids, out = [], []
    for r in range(logits.shape[0]):
        i, st = O.sample_from_logits(logits[r].astype(np.float64), int(states[r]), t, k, p)
        ids.append(i)
        out.append(st)
    return np.array(ids), np.array(out, dtype=np.uint32)


@pytest.mark.parametrize("vocab,rows", [(12, 64), (4096, 48), (32768, 12)])
@pytest.mark.parametrize("scale", [0.5, 3.0])
def test_sampler_matches_oracle(vocab, rows, scale):
    for n, (t, k, p) in enumerate(OPTS):
        lg = quantized_logits(vocab + n, rows, vocab, scale)
        st0 = np.array([O.mix_seed(11, n * 1000 + r) for r in range(rows)], dtype=np.uint32)
        st = st0.copy()
        got = pkg.sample_from_logits(lg, pkg.Sampling(t, k, p), st)
        want, want_st = oracle_rows(lg, st0, t, k, p)
        assert np.array_equal(st, want_st), (t, k, p)  # one draw per row, SeededRng arithmetic
        for r in np.nonzero(got != want)[0]:
            assert explainable(lg[r], t, k, p, int(st[r]), int(got[r])), (vocab, t, k, p, r, got[r], want[r])
        assert np.count_nonzero(got != want) <= max(1, rows // 50), (vocab, t, k, p)


def test_ties_follow_the_stable_sort():
    # all-equal logits: the stable descending sort keeps the lowest indices (Distribution.ts:67)
    lg = np.zeros((32, 10), np.float32)
    for t, k, p, keep in ((1.0, 5, 1.0, 5), (1.0, 0, 0.3, 3), (1.0, 0, 0.7, 7), (2.0, 4, 0.5, 2)):
        st0 = np.array([O.mix_seed(3, r) for r in range(32)], dtype=np.uint32)
        st = st0.copy()
        got = pkg.sample_from_logits(lg, pkg.Sampling(t, k, p), st)
        want, _ = oracle_rows(lg, st0, t, k, p)
        assert np.array_equal(got, want), (t, k, p)
        assert got.max() < keep


def test_greedy_rows_are_first_index_of_max():
    lg = np.array([[0, 3, 3, 1], [5, 5, 5, 5], [-1, -2, -0.5, -0.5]], np.float32)
    assert pkg.sample_from_logits(lg, pkg.GREEDY).tolist() == [1, 0, 2]


def test_generate_sampling_follows_step_logits():
    w = pkg.configs.MICROCHAT
    cfg = w.model
    params = pkg.init_params(cfg, w.weight_seed)
    n, new = 4, 12
    t, k, p = 0.9, 50, 0.9
    prompts = np.stack([O.uniform_ids(32, cfg.vocab_size, seed=900 + i) for i in range(n)])
    st0 = np.array([O.mix_seed(7 + i, 3) for i in range(n)], dtype=np.uint32)
    with pkg.Session(cfg, params, max_seqs=n) as sess:
        st = st0.copy()
        ids = sess.generate(prompts, new, pkg.Sampling(t, k, p), st)
        again = sess.generate(prompts, new, pkg.Sampling(t, k, p), st0.copy())
        assert np.array_equal(ids, again)  # same RNG states, same ids (CachedForward.Test.ts:81-87)
        for i in range(n):
            r = O.Rng(int(st0[i]))
            for _ in range(new):
                r.next_u32()
            assert int(r.state[0]) == int(st[i])  # one draw per new token
        top1 = sess.generate(prompts, new, pkg.Sampling(t, 1, 1.0), st0.copy())
        assert np.array_equal(top1, sess.generate(prompts, new))  # top-k 1 is the greedy argmax

        # replay the trajectory through shahd_step; the oracle sampler on the step logits must agree
        sess.prefill(list(range(n)), [pr[:-1] for pr in prompts])
        toks = [int(pr[-1]) for pr in prompts]
        states = [int(x) for x in st0]
        for s in range(new):
            logits, _ = sess.step(list(range(n)), toks)
            for i in range(n):
                want, states[i] = O.sample_from_logits(logits[i].astype(np.float64), states[i], t, k, p)
                if want != ids[i, s]:
                    assert explainable(logits[i], t, k, p, states[i], int(ids[i, s])), (i, s)
                toks[i] = int(ids[i, s])


@pytest.mark.parametrize("label,arch", ARCHS[:3], ids=[a[0] for a in ARCHS[:3]])
def test_generate_sampling_past_block_size(label, arch):
    cfg = pkg.ModelConfig(**arch)
    params = pkg.init_params(cfg, 5)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5]  # longer than BlockSize 8
    new = 2 * cfg.block_size + 3
    t, k, p = 1.0, 0, 0.8
    with pkg.Session(cfg, params, max_seqs=1) as sess:
        st = np.array([O.mix_seed(1, 3)], dtype=np.uint32)
        state = int(st[0])
        ids = sess.generate([prompt], new, pkg.Sampling(t, k, p), st)[0]
        dec = pkg.CachedDecoder(sess, prompt)
        for s in range(new):
            want, state = O.sample_from_logits(dec.logits.astype(np.float64), state, t, k, p)
            if want != ids[s]:
                assert explainable(dec.logits, t, k, p, state, int(ids[s])), s
            if s + 1 < new:
                dec.push(int(ids[s]))
        assert state == int(st[0])
