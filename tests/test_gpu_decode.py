"""GPU parity of the KV-cached decode path against the oracle (the reference's f64 forward on the same
f32 master weights). Tolerance (north_star): per-step logits within 2e-2 of the oracle's logit range
(bf16 weights, fp32 accumulation); greedy ids equal wherever the oracle's top-2 margin exceeds that.

Relations mirrored from Tests/CachedForward.Test.ts: every cached step vs the reference forward (:46-55),
the sliding window past BlockSize (:57-67), CachedGenerate ids (:69-78), input validation (:108-117),
MaxNewTokens = 0 (:128-132). Both projection regimes run: CUDA-core (SetScalarKernels(1)) and tcgen05
tiles (ShahdSetTensorCoreMinRows(1)).
"""
import numpy as np
import pytest

from tests.helpers import ARCHS, O, TOL_BF16, decode_loop, greedy_agrees, oracle_shape, pkg, range_rel_err

pytestmark = pytest.mark.gpu

BLOCK, VOCAB = 8, 12


@pytest.fixture(params=["simt", "umma"])
def regime(request):
    lib = pkg.load()
    if request.param == "simt":
        lib.SetScalarKernels(1)
    else:
        lib.ShahdSetTensorCoreMinRows(1)
    yield request.param
    lib.SetScalarKernels(0)


def build(arch, seed=1, max_seqs=4):
    cfg = pkg.ModelConfig(**arch)
    p = pkg.init_params(cfg, seed)
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    return cfg, pkg.Session(cfg, p, max_seqs=max_seqs), model


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_every_cached_step_matches_oracle(label, arch, regime):
    cfg, sess, model = build(arch)
    seq = [1, 5, 2, 8, 3, 0, 7, 11]
    cache = model.new_cache()
    for p, tok in enumerate(seq):
        want = cache.step(tok, p)
        logits, nxt = sess.step([0], [tok])
        assert sess.length(0) == p + 1
        assert range_rel_err(logits[0], want) < TOL_BF16
        assert greedy_agrees(nxt[0], want)
    assert pkg.load().ShahdDeviceErrorFlag() == 0


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_batched_ragged_rows_match_oracle(label, arch, regime):
    cfg, sess, model = build(arch)
    rng = O.Rng(23)
    prompts = [[int(rng.next_float() * VOCAB) for _ in range(n)] for n in (5, 1, 3)]
    sess.prefill([2, 0, 1], prompts)
    caches = []
    for pr in prompts:
        c = model.new_cache()
        c.prefill(pr)
        caches.append(c)
    slots = [2, 0, 1]
    for t in range(2):
        toks = [(3 * t + i) % VOCAB for i in range(3)]
        logits, nxt = sess.step(slots, toks)
        for i in range(3):
            want = caches[i].step(toks[i])
            assert range_rel_err(logits[i], want) < TOL_BF16
            assert greedy_agrees(nxt[i], want)


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_decoder_matches_oracle_past_blocksize(label, arch, regime):
    cfg, sess, model = build(arch)
    rng = O.Rng(17)
    seq = [int(rng.next_float() * VOCAB) for _ in range(3 * BLOCK + 2)]
    dec = pkg.CachedDecoder(sess, seq[:2])
    odec = O.Decoder(model, seq[:2])
    assert range_rel_err(dec.logits, odec.logits) < TOL_BF16
    for n in range(3, len(seq) + 1):
        dec.push(seq[n - 1])
        odec.push(seq[n - 1])
        assert sess.length(0) == odec.cache_length
        assert range_rel_err(dec.logits, odec.logits) < TOL_BF16


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_generate_greedy_ids_match_oracle(label, arch, regime):
    cfg, sess, model = build(arch)
    prompts = [[1, 5, 2], [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5]]  # the second is longer than BlockSize
    new = 2 * BLOCK + 3
    out = sess.generate(prompts, new)
    for prompt, ids in zip(prompts, out):
        # teacher-forced oracle along the GPU's own trajectory: every step must agree where decidable
        odec = O.Decoder(model, prompt)
        for k, tok in enumerate(ids):
            assert greedy_agrees(tok, odec.logits), (k, tok)
            odec.push(int(tok))
    # each sequence alone (CachedGenerate semantics per prompt) gives the same ids as in the batch
    alone = pkg.cached_generate(sess, prompts[1], new)
    assert alone[len(prompts[1]):] == out[1].tolist()


def test_generate_validation_and_zero_tokens():
    cfg, sess, model = build(ARCHS[2][1])
    with pytest.raises(pkg._lib.ShahdError, match="out of range"):
        sess.step([0], [VOCAB])
    with pytest.raises(pkg._lib.ShahdError, match="out of range"):
        sess.step([0], [-1])
    with pytest.raises(pkg._lib.ShahdError, match="listed twice"):
        sess.step([0, 0], [1, 2])
    with pytest.raises(pkg._lib.ShahdError, match="out of range"):
        sess.generate([[1, VOCAB]], 2)
    with pytest.raises(pkg._lib.ShahdError, match="empty prompt"):
        sess.generate([[1], []], 2)
    assert sess.length(0) == 0  # nothing half-appended by the rejected calls
    assert pkg.cached_generate(sess, [4, 2], 0) == [4, 2]
    sess.prefill([0], [[1, 2, 3, 4, 5, 6, 7, 8]])
    with pytest.raises(pkg._lib.ShahdError, match="window"):
        sess.step([0], [1])
    with pytest.raises(pkg._lib.ShahdError, match="capacity"):
        sess.prefill([0], [[1] * (BLOCK + 1)])


def test_gqa_cache_slots_and_reset():
    cfg, sess, model = build(ARCHS[3][1])
    sess.step([1], [3])
    assert sess.length(1) == 1 and sess.length(0) == 0
    sess.reset([1])
    assert sess.length(1) == 0


# ---- BASELINE shapes: spot parity at full model size ---------------------------------------------

def _teacher_forced_shape(workload, nseq, prompt_len, steps, regime_rows=None):
    cfg = workload.model
    p = pkg.init_params(cfg, workload.weight_seed)
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    sess = pkg.Session(cfg, p, max_seqs=nseq)
    prompts = [O.uniform_ids(prompt_len, cfg.vocab_size, seed=100 + i) for i in range(nseq)]
    sess.prefill(list(range(nseq)), [pr[:-1] for pr in prompts])
    decs = [O.Decoder(model, pr) for pr in prompts]
    toks = [int(pr[-1]) for pr in prompts]
    worst = 0.0
    for t in range(steps):
        logits, nxt = sess.step(list(range(nseq)), toks)
        for i in range(nseq):
            want = decs[i].logits
            worst = max(worst, range_rel_err(logits[i], want))
            assert greedy_agrees(nxt[i], want)
            toks[i] = int(nxt[i])
            decs[i].push(toks[i])
    assert worst < TOL_BF16, worst
    return worst


def test_microchat_shape_parity(regime):
    _teacher_forced_shape(pkg.configs.MICROCHAT, nseq=3, prompt_len=128, steps=24)


def test_foundry_shape_parity(regime):
    _teacher_forced_shape(pkg.configs.FOUNDRY, nseq=2, prompt_len=64, steps=24)


def test_phase2_shape_parity():
    _teacher_forced_shape(pkg.configs.PHASE2, nseq=2, prompt_len=16, steps=4)


def test_launch_modes_give_identical_ids():
    # programmatic dependent launch only changes scheduling: ids must be bit-identical with it off
    w = pkg.configs.MICROCHAT
    cfg = w.model
    p = pkg.init_params(cfg, w.weight_seed)
    prompts = np.stack([O.uniform_ids(40, cfg.vocab_size, seed=500 + i) for i in range(8)])
    lib = pkg.load()
    with decode_loop(False):  # the per-kernel step chain, where programmatic launch applies
        with pkg.Session(cfg, p, max_seqs=8) as sess:
            a = sess.generate(prompts, 20)
            lib.ShahdSetProgrammaticLaunch(0)
            try:
                b = sess.generate(prompts, 20)
            finally:
                lib.ShahdSetProgrammaticLaunch(1)
    assert np.array_equal(a, b)
    assert lib.ShahdDeviceErrorFlag() == 0


def test_decode_chains_agree_up_to_near_ties():
    # splitting the batch into concurrent chains changes tile shapes and attention splits, not the math:
    # a row may only diverge where the oracle's top-2 margin is within tolerance
    w = pkg.configs.MICROCHAT
    cfg = w.model
    p = pkg.init_params(cfg, w.weight_seed)
    prompts = np.stack([O.uniform_ids(96, cfg.vocab_size, seed=700 + i) for i in range(64)])
    lib = pkg.load()
    outs = {}
    with decode_loop(False):  # chains split the per-kernel step path
        with pkg.Session(cfg, p, max_seqs=64) as sess:
            for chains in (1, 2, 4):
                lib.ShahdSetDecodeChains(chains)
                outs[chains] = sess.generate(prompts, 24)
            lib.ShahdSetDecodeChains(0)
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    for chains in (2, 4):
        for i in np.nonzero((outs[chains] != outs[1]).any(axis=1))[0][:4]:
            k = int(np.argmax(outs[chains][i] != outs[1][i]))
            odec = O.Decoder(model, prompts[i])
            for t in outs[1][i][:k]:
                odec.push(int(t))
            lg = odec.logits
            s = np.sort(lg)
            assert s[-1] - s[-2] <= TOL_BF16 * (lg.max() - lg.min()), (chains, i, k)


def test_microchat_generate_spot_check_and_determinism():
    w = pkg.configs.MICROCHAT
    cfg = w.model
    p = pkg.init_params(cfg, w.weight_seed)
    sess = pkg.Session(cfg, p, max_seqs=w.seqs)
    prompts = np.stack([O.uniform_ids(w.prompt_len, cfg.vocab_size, seed=1000 + i) for i in range(w.seqs)])
    out1 = sess.generate(prompts, 64)
    for _ in range(4):  # deterministic run to run (host staging rows and prefill plans do not race)
        assert np.array_equal(out1, sess.generate(prompts, 64))
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    for i in (0, 37):
        odec = O.Decoder(model, prompts[i])
        for k, tok in enumerate(out1[i][:32]):
            assert greedy_agrees(tok, odec.logits), (i, k)
            odec.push(int(tok))


def test_decode_loop_agrees_with_per_kernel_path():
    # greedy generate runs its decode steps as per-kernel launch chains by default; with the persistent cluster
    # loop on, the same steps run in one launch (different tiles, reduction order and attention split). Both
    # must pass the oracle's teacher-forced check, and may only differ from one another at near ties.
    w = pkg.configs.MICROCHAT
    cfg = w.model
    p = pkg.init_params(cfg, w.weight_seed)
    prompts = np.stack([O.uniform_ids(64, cfg.vocab_size, seed=300 + i) for i in range(40)])
    lib = pkg.load()
    res = {}
    for mode in (1, 0):
        with decode_loop(mode == 1):
            with pkg.Session(cfg, p, max_seqs=40) as sess:
                res[mode] = sess.generate(prompts, 24)
    assert lib.ShahdDeviceErrorFlag() == 0
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    for mode in (0, 1):
        chk = model.check_trajectories(prompts, res[mode], TOL_BF16)
        assert int(chk["fails"].sum()) == 0, (mode, np.nonzero(chk["fails"])[0][:4])


def test_fused_attention_shape_parity():
    # the FusedAttention config's attention shape: 8 query heads over 2 kv heads (GQA 4), head_dim 64,
    # RoPE base 10000, causal prefill of 511 positions then cached decode steps to the end of a 512 window
    cfg = pkg.ModelConfig(embed_dim=512, num_layers=1, num_heads=8, kv_heads=2, block_size=512, vocab_size=512,
                          mlp_hidden=1024, position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu")
    w = pkg.configs.Workload("attention", cfg, weight_seed=3, seqs=2, prompt_len=512, new_tokens=0)
    worst = _teacher_forced_shape(w, nseq=2, prompt_len=508, steps=4)
    assert worst < TOL_BF16
