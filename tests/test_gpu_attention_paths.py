"""Decode-row attention launch shapes against the oracle (CachedForward.ts:76-84 per row), on each of the
three decode attention kernels.

The decode attention picks its launch from the step's rows and kv heads: one CTA per (row, kv head) when
they fill the GPU, position splits merged through partials when they leave SMs idle. Each case below
lands on a different combination of head_dim, query heads per kv head (G), split count and grid size
(more CTAs than fit at once included); every row's teacher-forced logits are checked over a page
boundary and ragged lengths.
"""
import numpy as np
import pytest

from tests.helpers import O, TOL_BF16, greedy_agrees, oracle_shape, pkg, range_rel_err

pytestmark = pytest.mark.gpu

CASES = [
    # label, model, rows
    ("d128 G1 Hk2, 160 rows (more CTAs than one wave)", dict(embed_dim=256, num_heads=2, kv_heads=2), 160),
    ("d32 G8 Hk1, 20 rows (position splits)", dict(embed_dim=256, num_heads=8, kv_heads=1), 20),
    ("d64 G2 Hk2, 80 rows (one split per row)", dict(embed_dim=256, num_heads=4, kv_heads=2), 80),
    ("d64 G1 Hk8, 40 rows (eight kv heads)", dict(embed_dim=512, num_heads=8, kv_heads=8), 40),
]


# 0: the automatic choice (read-ahead rows kernel at these lengths), 2: the page-ring kernel, 3: the
# page-streaming kernel (producer warp, one page per compute warp)
KERNELS = {"auto": 0, "page ring": 2, "page streaming": 3}


@pytest.fixture
def decode_attention_kernel(request):
    lib = pkg.load()
    lib.ShahdSetDecodeAttentionKernel(KERNELS[request.param])
    yield request.param
    lib.ShahdSetDecodeAttentionKernel(0)


@pytest.mark.parametrize("decode_attention_kernel", list(KERNELS), indirect=True)
@pytest.mark.parametrize("label,arch,rows", CASES, ids=[c[0] for c in CASES])
def test_decode_attention_paths_match_oracle(label, arch, rows, decode_attention_kernel):
    cfg = pkg.ModelConfig(num_layers=2, block_size=128, vocab_size=256, mlp_hidden=2 * arch["embed_dim"],
                          position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu", **arch)
    p = pkg.init_params(cfg, 11)
    model = O.Model(oracle_shape(cfg, "F32"), p.astype(np.float64))
    sess = pkg.Session(cfg, p, max_seqs=rows)
    # ragged prompts that straddle the 64-position page and 32-position task boundaries
    prompts = [O.uniform_ids(30 + (7 * i) % 70, cfg.vocab_size, seed=900 + i) for i in range(rows)]
    sess.prefill(list(range(rows)), [pr[:-1] for pr in prompts])
    decs = [O.Decoder(model, pr) for pr in prompts]
    toks = [int(pr[-1]) for pr in prompts]
    worst = 0.0
    for _ in range(3):
        logits, nxt = sess.step(list(range(rows)), toks)
        for i in range(rows):
            want = decs[i].logits
            worst = max(worst, range_rel_err(logits[i], want))
            assert greedy_agrees(nxt[i], want), (label, i)
            toks[i] = int(nxt[i])
            decs[i].push(toks[i])
    assert worst < TOL_BF16, (label, worst)
    assert pkg.load().ShahdDeviceErrorFlag() == 0
