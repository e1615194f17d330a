"""The reference's relational tests, ported onto the CPU oracle (pins the restatement).

Mirrors Tests/CachedForward.Test.ts (cached step vs full forward, sliding window, CachedGenerate ids ==
Generate ids, stochastic same-RNG equality, validation, GQA slots, MaxNewTokens=0) and
Tests/SeededRng.Test.ts. Model seed = Training.Seed default 1 (Brain/Config/Constants.ts:48) through
CreateRngStreams(seed).InitRng, as CachedForward.Test.ts:27-30 builds its models.
"""
import numpy as np
import pytest

from oracle import oracle as O

LOGIT_TOL = 1e-9  # CachedForward.Test.ts:11
BLOCK = 8
VOCAB = 12
GREEDY = dict(temperature=0.0, top_k=0, top_p=1.0)
SHARED = dict(embed_dim=16, num_layers=2, block_size=BLOCK, vocab_size=VOCAB, mlp_hidden=32)  # MlpRatio 2

# CachedForward.Test.ts:18-25
ARCHS = [
    ("Learned/LayerNorm/Relu/MHA", dict(SHARED, num_heads=2)),
    ("Learned/LayerNorm/Relu/MHA untied", dict(SHARED, num_heads=1, weight_tying=False)),
    ("Rope/RmsNorm/SwiGlu/MHA", dict(SHARED, num_heads=4, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")),
    ("Rope/RmsNorm/SwiGlu/GQA 2-of-4",
     dict(SHARED, num_heads=4, kv_heads=2, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")),
    ("Rope/LayerNorm/Relu", dict(SHARED, num_heads=2, position_scheme="Rope")),
    ("Learned/RmsNorm/GeGlu/GQA 1-of-2", dict(SHARED, num_heads=2, kv_heads=1, norm_kind="RmsNorm", mlp_kind="GeGlu")),
]


def build(arch: dict, precision: str = "F64") -> O.Model:
    shape = O.Shape(precision=precision, **arch)
    return O.Model(shape, O.init_params(shape, seed=1))


def full_last_row(model: O.Model, ids) -> np.ndarray:
    return model.forward(list(ids)[-BLOCK:])[-1]


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_every_cached_step_matches_full_forward_row(label, arch):
    model = build(arch)
    seq = [1, 5, 2, 8, 3, 0, 7, 11]
    full = model.forward(seq)
    cache = model.new_cache()
    for p, tok in enumerate(seq):
        logits = cache.step(tok, p)
        assert np.max(np.abs(logits - full[p])) < LOGIT_TOL


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_decoder_matches_sliding_window_forward(label, arch):
    model = build(arch)
    rng = O.Rng(17)
    seq = [int(rng.next_float() * VOCAB) for _ in range(3 * BLOCK + 2)]
    dec = O.Decoder(model, seq[:2])
    assert np.max(np.abs(dec.logits - full_last_row(model, seq[:2]))) < LOGIT_TOL
    for n in range(3, len(seq) + 1):
        dec.push(seq[n - 1])
        assert np.max(np.abs(dec.logits - full_last_row(model, seq[:n]))) < LOGIT_TOL


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_cached_generate_equals_generate_greedy(label, arch):
    model = build(arch)
    for prompt in ([1, 5, 2], [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5]):
        new = 2 * BLOCK + 3
        unc, _ = model.generate(prompt, new, **GREEDY)
        cac, _ = model.cached_generate(prompt, new, **GREEDY)
        assert len(cac) == len(prompt) + new
        assert list(cac) == list(unc)


def test_cached_generate_matches_generate_stochastic():
    model = build(ARCHS[3][1])
    opts = dict(temperature=0.9, top_k=5, top_p=0.9)
    unc, s1 = model.generate([2, 7], 20, rng_state=5, **opts)
    cac, s2 = model.cached_generate([2, 7], 20, rng_state=5, **opts)
    assert list(cac) == list(unc) and s1 == s2


def test_empty_prompt_rejected():
    model = build(ARCHS[0][1])
    with pytest.raises(O.OracleError, match="empty prompt"):
        model.generate([], 3)
    with pytest.raises(O.OracleError, match="empty prompt"):
        model.cached_generate([], 3)


def test_cached_path_validates_ids_and_positions():
    model = build(ARCHS[2][1])
    cache = model.new_cache()
    with pytest.raises(O.OracleError, match="out of range"):
        cache.step(VOCAB, 0)
    with pytest.raises(O.OracleError, match="out of range"):
        cache.step(-1, 0)
    with pytest.raises(O.OracleError, match="contiguous"):
        cache.step(1, 3)
    with pytest.raises(O.OracleError, match="out of range"):
        model.cached_generate([1, VOCAB], 2)
    assert cache.length == 0


def test_gqa_cache_holds_one_slot_per_kv_head():
    model = build(ARCHS[3][1])
    cache = model.new_cache()
    cache.step(3, 0)
    k, v = cache.read(0, 1)
    assert k.shape == (1, 4)
    with pytest.raises(O.OracleError):
        cache.read(0, 2)


def test_max_new_tokens_zero_returns_prompt():
    model = build(ARCHS[0][1])
    assert list(model.cached_generate([4, 2], 0)[0]) == [4, 2]
    assert list(model.generate([4, 2], 0)[0]) == [4, 2]


@pytest.mark.parametrize("label,arch", ARCHS[2:4], ids=[a[0] for a in ARCHS[2:4]])
def test_f32_storage_cached_matches_full_forward(label, arch):
    # F32 storage rounds every tensor op's output, the cached row math stays f64: agreement to f32 noise.
    model = build(arch, precision="F32")
    seq = [1, 5, 2, 8, 3, 0, 7, 11]
    full = model.forward(seq)
    cache = model.new_cache()
    for p, tok in enumerate(seq):
        assert np.max(np.abs(cache.step(tok, p) - full[p])) < 1e-5


def test_prefill_then_step_equals_steps():
    model = build(ARCHS[3][1])
    seq = [4, 9, 1, 1, 0, 6]
    a = model.new_cache()
    for p, t in enumerate(seq[:-1]):
        a.step(t, p)
    la = a.step(seq[-1])
    b = model.new_cache()
    b.prefill(seq[:-1])
    lb = b.step(seq[-1])
    assert np.max(np.abs(la - lb)) < LOGIT_TOL
    for layer in range(2):
        for g in range(2):
            ka, va = a.read(layer, g)
            kb, vb = b.read(layer, g)
            assert np.max(np.abs(ka - kb)) < LOGIT_TOL and np.max(np.abs(va - vb)) < LOGIT_TOL


# ---- Tests/SeededRng.Test.ts ------------------------------------------------------------------

def test_rng_reproducible_and_in_unit_interval():
    a, b = O.Rng(42), O.Rng(42)
    for _ in range(100):
        x = a.next_float()
        assert x == b.next_float() and 0 <= x < 1


def test_rng_streams_independent():
    s1 = O.create_streams(7)
    r = O.Rng(s1[0])
    for _ in range(1000):
        r.next_float()
    d1 = O.Rng(s1[1])
    s2 = O.create_streams(7)
    d2 = O.Rng(s2[1])
    assert [d1.next_float() for _ in range(3)] == [d2.next_float() for _ in range(3)]
    assert O.Rng(s1[0]).next_float() != O.Rng(s1[1]).next_float()


def _mix_seed_py(seed: int, stream: int) -> int:
    m = 0xFFFFFFFF
    x = (seed ^ (((stream + 1) * 0x9E3779B9) & m)) & m
    x = ((x ^ (x >> 16)) * 0x45D9F3B) & m
    x = ((x ^ (x >> 16)) * 0x45D9F3B) & m
    return (x ^ (x >> 16)) & m


def test_rng_matches_independent_python_restatement():
    # SeededRng.ts:7-12 (MixSeed) and :32-40 (LCG) restated in Python integers.
    for seed in (0, 1, 7, 123456789, 0xFFFFFFFF):
        for stream in range(4):
            assert O.mix_seed(seed, stream) == _mix_seed_py(seed, stream)
    st = 42
    r = O.Rng(42)
    for _ in range(50):
        st = (st * 1664525 + 1013904223) & 0xFFFFFFFF
        assert r.next_u32() == st
    assert O.Rng(42).next_float() == ((42 * 1664525 + 1013904223) & 0xFFFFFFFF) / 4294967296.0
