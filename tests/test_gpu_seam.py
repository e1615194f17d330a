"""GPU parity of the matmul-level seam against the oracle (and the reference's edge shapes).

Mirrors Tests/Compute.Test.ts:109-145 (GoFfi vs TS, f64 1e-10 relative), :147-221 and :275-313 (Into /
NtAcc / TnAcc accumulate semantics, NtInto on dirty buffers) and Tests/FfiGuard.Test.ts:146-200
(f64 1e-10 / f32 1e-4 scaled error), plus the tensor-core bf16 MatMulNT on the operator-sweep shapes.
"""
import numpy as np
import pytest

from tests.helpers import O, pkg

pytestmark = pytest.mark.gpu

SHAPES_F64 = [(256, 128, 512), (7, 5, 3), (13, 128, 9), (16, 13, 5), (1, 1, 1)]
SHAPES_NT = [(33, 70, 19), (7, 5, 3), (1, 1, 1)]


@pytest.fixture(scope="module")
def gpu():
    return pkg.GpuBackend()


def scaled(got, want):
    return float(np.max(np.abs(want - got) / np.maximum(np.abs(want), 1)))


@pytest.mark.parametrize("m,k,n", SHAPES_F64)
def test_matmul_f64_matches_oracle(gpu, m, k, n):
    rng = np.random.default_rng(9)
    a = rng.standard_normal(m * k)
    b = rng.standard_normal(k * n)
    got = gpu.MatMul(a, b, m, k, n)
    want = O.matmul(a.reshape(m, k), b.reshape(k, n)).ravel()
    assert np.max(np.abs(want - got) / (np.abs(want) + 1e-9)) < 1e-10


def test_known_answers(gpu):
    out = np.full(4, 7.0)
    gpu.MatMulNtInto(np.array([1, 2, 3, 4, 5, 6.0]), np.array([1, 0, -1, 2, 1, 0.0]), out, 2, 3, 2)
    assert out.tolist() == [-2, 4, -2, 13]
    assert gpu.MatMul(np.array([1, 2, 3, 4.0]), np.array([1, 0, 0, 1.0]), 2, 2, 2).tolist() == [1, 2, 3, 4]


@pytest.mark.parametrize("m,k,n", SHAPES_NT)
@pytest.mark.parametrize("dt,tol", [(np.float64, 1e-10), (np.float32, 1e-4)])
def test_into_ntacc_tnacc_semantics(gpu, m, k, n, dt, tol):
    rng = np.random.default_rng(21)
    a = rng.standard_normal((m, k)).astype(dt)
    b = rng.standard_normal((k, n)).astype(dt)
    bt = rng.standard_normal((n, k)).astype(dt)
    dout = rng.standard_normal((m, n)).astype(dt)
    seed = rng.standard_normal((m, n)).astype(dt)
    dbseed = rng.standard_normal((k, n)).astype(dt)
    f = lambda x: x.astype(np.float64)  # noqa: E731

    into = np.full(m * n, 7, dtype=dt)
    gpu.MatMulInto(a.ravel(), b.ravel(), into, m, k, n)
    assert scaled(into, O.matmul(f(a), f(b)).ravel()) < tol

    nt_want = O.matmul_nt(f(a), f(bt))
    nt = np.full(m * n, 7, dtype=dt)
    gpu.MatMulNtInto(a.ravel(), bt.ravel(), nt, m, k, n)
    assert scaled(nt, nt_want.ravel()) < tol

    acc = seed.ravel().copy()
    gpu.MatMulNtAcc(a.ravel(), bt.ravel(), acc, m, k, n)
    assert scaled(acc, (nt_want + f(seed)).ravel()) < tol

    db = dbseed.ravel().copy()
    gpu.MatMulTnAcc(a.ravel(), dout.ravel(), db, m, k, n)
    assert scaled(db, (O.matmul_tn(f(a), f(dout)) + f(dbseed)).ravel()) < tol


def test_seam_validates_before_native_memory(gpu):
    ok = lambda s: np.zeros(s)  # noqa: E731
    with pytest.raises(ValueError, match="MatMulInto"):
        gpu.MatMulInto(np.zeros(3), ok(12), ok(8), 2, 3, 4)
    with pytest.raises(TypeError, match="mixed"):
        gpu.MatMul(ok(6), np.zeros(12, np.float32), 2, 3, 4)
    with pytest.raises(ValueError, match="empty"):
        gpu.MatMulNtAcc(ok(6), ok(12), np.zeros(0), 2, 3, 4)
    with pytest.raises(ValueError, match="dimension M"):
        gpu.MatMulInto(ok(1), ok(1), ok(1), 0, 1, 1)


# ---- tcgen05 bf16 MatMulNT on device operands -----------------------------------------------------

SWEEP = [(1, 256, 768), (64, 256, 1024), (64, 1024, 256), (130, 256, 4096), (1024, 1024, 4096), (200, 40, 72),
         (8192, 256, 768)]


@pytest.mark.parametrize("m,k,n", SWEEP)
def test_bf16_tensor_core_matmul_nt(m, k, n):
    import torch
    g = torch.Generator(device="cpu").manual_seed(2)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    bt = torch.randn(n, k, generator=g).to(torch.bfloat16).cuda()
    out = torch.full((m, n), 7.0, device="cuda")
    pkg.backend.matmul_nt_bf16_device(a.data_ptr(), bt.data_ptr(), out.data_ptr(), m, k, n, acc=False)
    torch.cuda.synchronize()
    ref = a.double() @ bt.double().T
    rng = float(ref.max() - ref.min())
    err = float((out.double() - ref).abs().max()) / rng
    assert err < 1e-4, err  # fp32 accumulation of exact bf16 products: order-only differences
    seed = torch.randn(m, n, generator=g).cuda()
    acc = seed.clone()
    pkg.backend.matmul_nt_bf16_device(a.data_ptr(), bt.data_ptr(), acc.data_ptr(), m, k, n, acc=True)
    torch.cuda.synchronize()
    err = float((acc.double() - (ref + seed.double())).abs().max()) / rng
    assert err < 1e-4, err
    assert pkg._lib.load().ShahdDeviceErrorFlag() == 0


# ---- f32 seam on the tensor cores (split-TF32, three tcgen05 kind::tf32 passes) ---------------------
# The operator-sweep shapes of the MatMulNT config: fp32 A[M,K], B[N,K] ~ N(0,1); M >= 64 takes the
# tensor cores, M = 1 the CUDA-core kernel. The bar is north_star's: within 1e-4 of the output range for
# TF32/fp32. (FfiGuard's max(|want|, 1)-scaled 1e-4, Tests/FfiGuard.Test.ts:146-200, is a bar for exact fp32
# FMA chains; its shapes all have fewer than 64 rows and keep the CUDA-core kernel, which SetScalarKernels
# forces, as the reference's test does.) Reference: an f64 product of the same f32 inputs (numpy's f64
# matmul for the large shapes: the oracle's f64 dot product, only faster).

SWEEP_NK = [(768, 256), (1024, 256), (256, 1024), (4096, 256), (4096, 1024)]


def range_err(got, want):
    return float(np.abs(got - want).max()) / float(want.max() - want.min())


@pytest.mark.parametrize("m", [1, 64, 1024])
@pytest.mark.parametrize("n,k", SWEEP_NK)
def test_f32_matmul_nt_sweep_shapes(gpu, m, n, k):
    rng = np.random.default_rng(2)
    a = rng.standard_normal((m, k), dtype=np.float32)
    bt = rng.standard_normal((n, k), dtype=np.float32)
    want = a.astype(np.float64) @ bt.astype(np.float64).T
    out = np.full(m * n, 7, np.float32)
    gpu.MatMulNtInto(a.ravel(), bt.ravel(), out, m, k, n)
    assert range_err(out.reshape(m, n), want) < 1e-4
    seed = rng.standard_normal(m * n).astype(np.float32)
    acc = seed.copy()
    gpu.MatMulNtAcc(a.ravel(), bt.ravel(), acc, m, k, n)
    assert range_err(acc, want.ravel() + seed) < 1e-4


def test_f32_matmul_nt_largest_sweep_shape(gpu):
    m, n, k = 8192, 4096, 1024
    rng = np.random.default_rng(2)
    a = rng.standard_normal((m, k), dtype=np.float32)
    bt = rng.standard_normal((n, k), dtype=np.float32)
    out = np.empty(m * n, np.float32)
    gpu.MatMulNtInto(a.ravel(), bt.ravel(), out, m, k, n)
    want = a.astype(np.float64) @ bt.astype(np.float64).T
    assert range_err(out.reshape(m, n), want) < 1e-4


@pytest.mark.parametrize("m,k,n", [(64, 256, 768), (300, 100, 130), (1024, 1024, 256)])
def test_f32_matmul_nn_on_tensor_cores(gpu, m, k, n):
    rng = np.random.default_rng(4)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    out = np.full(m * n, 7, np.float32)
    gpu.MatMulInto(a.ravel(), b.ravel(), out, m, k, n)
    assert range_err(out.reshape(m, n), a.astype(np.float64) @ b.astype(np.float64)) < 1e-4
    assert pkg._lib.load().ShahdDeviceErrorFlag() == 0


def test_scalar_kernels_force_exact_fp32_chains(gpu):
    # SetScalarKernels(1) (matmul.go:111-118) forces the CUDA-core kernel: FfiGuard's scaled bar then holds at
    # tensor-core-sized shapes too
    m, k, n = 256, 128, 512
    rng = np.random.default_rng(6)
    a = rng.standard_normal((m, k), dtype=np.float32)
    bt = rng.standard_normal((n, k), dtype=np.float32)
    out = np.empty(m * n, np.float32)
    gpu.SetScalarKernels(True)
    try:
        gpu.MatMulNtInto(a.ravel(), bt.ravel(), out, m, k, n)
    finally:
        gpu.SetScalarKernels(False)
    assert scaled(out, (a.astype(np.float64) @ bt.astype(np.float64).T).ravel()) < 1e-4


@pytest.mark.parametrize("m,k,n", [(64, 256, 768), (1024, 1024, 4096), (200, 40, 72)])
def test_f32_device_tensor_core_matmul_nt(m, k, n):
    import torch
    g = torch.Generator(device="cpu").manual_seed(2)
    a = torch.randn(m, k, generator=g).cuda()
    bt = torch.randn(n, k, generator=g).cuda()
    a0, b0 = a.clone(), bt.clone()
    out = torch.full((m, n), 7.0, device="cuda")
    pkg.backend.matmul_nt_f32_device(a.data_ptr(), bt.data_ptr(), out.data_ptr(), m, k, n, acc=False)
    torch.cuda.synchronize()
    ref = a.double() @ bt.double().T
    rng = float(ref.max() - ref.min())
    assert float((out.double() - ref).abs().max()) / rng < 1e-4
    assert torch.equal(a, a0) and torch.equal(bt, b0)  # the operands are not modified
    seed = torch.randn(m, n, generator=g).cuda()
    acc = seed.clone()
    pkg.backend.matmul_nt_f32_device(a.data_ptr(), bt.data_ptr(), acc.data_ptr(), m, k, n, acc=True)
    torch.cuda.synchronize()
    assert float((acc.double() - (ref + seed.double())).abs().max()) / rng < 1e-4
    assert pkg._lib.load().ShahdDeviceErrorFlag() == 0
