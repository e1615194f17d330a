"""The FusedAttention operator (shahd_attention_*: RoPE, causal prefill, then 1-token decode steps over the
paged cache) against the oracle's restatement (MultiHeadAttention.ts:46-74 core, CausalSoftmax.ts:17-33,
AttendRow CachedRowMath.ts:60-86): every prefill row and every decode step of the checked sequences, within
2e-2 of the oracle output's range (the bf16 bar: K/V rows are stored in bf16; the tensor-core prefill also
rounds Q and P to bf16). Covers the FusedAttention configuration (8 query heads over 2 kv heads, head_dim 64,
RoPE base 10000, prompts of 512, 256 sequences), both prefill kernels, the three decode kernels, and other
head shapes."""
import numpy as np
import pytest

from tests.helpers import O, pkg

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 2e-2


def _qkv(n, T, H, Hk, d, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, T, H, d), dtype=np.float32), rng.standard_normal((n, T, Hk, d), dtype=np.float32),
            rng.standard_normal((n, T, Hk, d), dtype=np.float32))


def _run(n, T, steps, H, Hk, d, base, seed, max_seqs=None):
    """Prefill T positions of n sequences, then `steps` decode steps; returns (q, k, v, prefill out, decode outs)."""
    q, k, v = _qkv(n, T + steps, H, Hk, d, seed)
    dev = torch.device("cuda", 0)
    # the copies and the calls share one stream (not the legacy default stream, which a stream argument of 0
    # does not name: 0 selects the operator's own stream), so the calls see the copied inputs and torch
    # reuses no tensor that a pending call still reads
    ts = torch.cuda.Stream(device=dev)
    cs = ts.cuda_stream
    with torch.cuda.stream(ts), pkg.FusedAttention(max_seqs or n, H, Hk, d, T + steps, base) as op:
        tq = torch.from_numpy(np.ascontiguousarray(q[:, :T])).to(dev)
        tk = torch.from_numpy(np.ascontiguousarray(k[:, :T])).to(dev)
        tv = torch.from_numpy(np.ascontiguousarray(v[:, :T])).to(dev)
        out = torch.empty((n, T, H, d), dtype=torch.float32, device=dev)
        op.prefill(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), n, T, out.data_ptr(), cs)
        dec = []
        for s in range(steps):
            sq = torch.from_numpy(np.ascontiguousarray(q[:, T + s])).to(dev)
            sk = torch.from_numpy(np.ascontiguousarray(k[:, T + s])).to(dev)
            sv = torch.from_numpy(np.ascontiguousarray(v[:, T + s])).to(dev)
            o = torch.empty((n, H, d), dtype=torch.float32, device=dev)
            op.decode(sq.data_ptr(), sk.data_ptr(), sv.data_ptr(), n, o.data_ptr(), cs)
            dec.append(o)
        torch.cuda.synchronize()
        assert op.length(0) == T + steps
        pre = out.cpu().numpy()
        dec = np.stack([o.cpu().numpy() for o in dec], axis=1) if steps else None
    assert pkg.load().ShahdDeviceErrorFlag() == 0
    return q, k, v, pre, dec


def _check(q, k, v, pre, dec, base, seqs):
    T = pre.shape[1]
    worst = 0.0
    for i in seqs:
        want = O.fused_attention(q[i], k[i], v[i], base)  # [T + steps, H, d]
        rng = float(want.max() - want.min())
        worst = max(worst, float(np.abs(pre[i] - want[:T]).max()) / rng)
        if dec is not None:
            worst = max(worst, float(np.abs(dec[i] - want[T:]).max()) / rng)
    assert worst < TOL, worst
    return worst


@pytest.fixture
def kernels(request):
    lib = pkg.load()
    umma, decode_kernel = request.param
    lib.ShahdSetTensorCorePrefillAttention(umma)
    lib.ShahdSetDecodeAttentionKernel(decode_kernel)
    yield request.param
    lib.ShahdSetTensorCorePrefillAttention(1)
    lib.ShahdSetDecodeAttentionKernel(0)


@pytest.mark.parametrize("kernels", [(1, 0), (0, 1), (1, 2), (1, 3)], indirect=True,
                         ids=["tensor-core prefill, auto decode", "CUDA-core prefill, rows decode",
                              "tensor-core prefill, page-ring decode", "tensor-core prefill, page-streaming decode"])
def test_fused_attention_config_heads_prefill_512_then_decode(kernels):
    q, k, v, pre, dec = _run(n=6, T=512, steps=12, H=8, Hk=2, d=64, base=10000.0, seed=3)
    _check(q, k, v, pre, dec, 10000.0, range(6))


def test_fused_attention_256_sequences():
    # the configuration's sequence count: grids larger than one wave, the automatic decode kernel at length 512+
    q, k, v, pre, dec = _run(n=256, T=512, steps=4, H=8, Hk=2, d=64, base=10000.0, seed=3)
    _check(q, k, v, pre, dec, 10000.0, (0, 101, 255))


@pytest.mark.parametrize("shape", [(4, 4, 32), (8, 1, 64), (4, 2, 128), (16, 2, 64)],
                         ids=["d32 G1", "d64 G8", "d128 G2", "d64 G8 Hk2"])
def test_fused_attention_other_head_shapes(shape):
    H, Hk, d = shape
    q, k, v, pre, dec = _run(n=5, T=130, steps=70, H=H, Hk=Hk, d=d, base=10000.0, seed=9)
    _check(q, k, v, pre, dec, 10000.0, range(5))


def test_fused_attention_without_rope_and_short_prompts():
    q, k, v, pre, dec = _run(n=3, T=1, steps=66, H=4, Hk=2, d=64, base=0.0, seed=11, max_seqs=7)
    _check(q, k, v, pre, dec, 0.0, range(3))


def test_fused_attention_rejects_bad_arguments():
    with pytest.raises(pkg._lib.ShahdError):
        pkg.FusedAttention(4, 6, 4, 64, 128)  # kv heads must divide the query heads
    with pkg.FusedAttention(2, 4, 2, 64, 16) as op:
        with pytest.raises(pkg._lib.ShahdError):
            op.prefill(1, 1, 1, 3, 8, 1)  # more sequences than the operator holds
        with pytest.raises(pkg._lib.ShahdError):
            op.prefill(1, 1, 1, 1, 17, 1)  # longer than its capacity
