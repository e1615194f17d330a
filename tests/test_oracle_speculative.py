"""The oracle's SpeculativeSample restatement against the reference's own relations
(Tests/SpeculativeSampling.Test.ts): a full sequence is produced; a draft equal to the target accepts every
proposal (q == p, acceptance probability 1) in fewer target passes than tokens; a weaker draft still yields
a full valid sequence; and one round on given logits uses the Rng exactly like the reference's loop
(one draw per examined proposal, one for the residual or bonus)."""
import numpy as np

from oracle import oracle as O

TINY = dict(vocab_size=20, embed_dim=16, num_heads=2, block_size=32, mlp_hidden=64)


def _model(layers, seed):
    shape = O.Shape(num_layers=layers, **TINY)
    return O.Model(shape, O.init_params(shape, seed))


def test_full_sequence_and_identical_draft_accepts_everything():
    m = _model(2, 5)
    ids, _, stats = O.speculative_sample(m, m, [1, 2, 3], 12, rng_state=3, temperature=0.9, top_k=8, top_p=0.95)
    assert len(ids) == 3 + 12
    calls, drafted, accepted = stats
    assert accepted == drafted
    assert calls < 12


def test_weaker_draft_full_valid_sequence():
    t, d = _model(2, 7), _model(1, 11)
    ids, _, stats = O.speculative_sample(t, d, [4, 5, 6], 10, rng_state=2, temperature=1.0, top_k=10, top_p=0.95)
    assert len(ids) == 13 and all(0 <= i < 20 for i in ids)
    assert stats[2] <= stats[1]


def test_round_draw_accounting():
    rng = np.random.default_rng(0)
    V, g = 16, 3
    tl = rng.standard_normal((g + 1, V))
    dl = tl[:g].copy()  # the draft agrees exactly: all proposals accepted, then a bonus draw
    prop = [int(np.argmax(r)) for r in dl]
    ids, acc, st = O.speculative_round(tl, dl, prop, budget=10, rng_state=9, temperature=1.0)
    assert acc == g and ids[:g] == prop and len(ids) == g + 1
    r = O.Rng(9)
    for _ in range(g + 1):
        r.next_u32()
    assert st == r.state[0]
    # budget reached by the accepted proposals: no bonus draw
    ids, acc, st = O.speculative_round(tl, dl, prop, budget=g, rng_state=9, temperature=1.0)
    assert len(ids) == g and acc == g
    r = O.Rng(9)
    for _ in range(g):
        r.next_u32()
    assert st == r.state[0]


def test_rejected_proposal_is_replaced_from_the_residual():
    V = 8
    tl = np.full((2, V), -30.0)
    tl[0, 3] = 0.0  # the target puts all its mass on id 3
    dl = np.full((1, V), -30.0)
    dl[0, 5] = 0.0  # the draft proposes id 5, which the target never picks
    ids, acc, _ = O.speculative_round(tl, dl, [5], budget=4, rng_state=1, temperature=1.0)
    assert acc == 0 and ids == [3]
