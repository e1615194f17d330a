"""Known answers and reference-kernel agreement for the oracle's matmul and sampling semantics.

Goldens: MatMulNT 2x3 (Tests/MatMulNT.Test.ts:43-52), identity multiply (Tests/Compute.Test.ts:271-272),
the top-k/top-p worked example (Brain/Sampling/Distribution.ts:61-64). The reference's own C kernels
(GoKernels/ffi/matmul_*.c, built into oracle/_ref by oracle/Makefile) check the oracle's matmul on the
edge shapes of Tests/Compute.Test.ts:109-145 and :275-313 and Tests/FfiGuard.Test.ts:146-200.
"""
import ctypes
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_matmul_nt_known_answer():
    a = np.array([[1, 2, 3], [4, 5, 6]], dtype=np.float64)
    b = np.array([[1, 0, -1], [2, 1, 0]], dtype=np.float64)
    assert O.matmul_nt(a, b).ravel().tolist() == [-2, 4, -2, 13]


def test_identity_multiply():
    out = O.matmul(np.array([[1, 2], [3, 4]], np.float64), np.array([[1, 0], [0, 1]], np.float64))
    assert out.ravel().tolist() == [1, 2, 3, 4]


def test_matmul_nt_equals_matmul_of_transpose():
    # MatMulNT.Test.ts:75-96: bit-identical to MatMul(A, Transpose(B)) in f64 (no zero entries here).
    rng = np.random.default_rng(3)
    a = rng.standard_normal((7, 5))
    bt = rng.standard_normal((3, 5))
    assert np.array_equal(O.matmul_nt(a, bt), O.matmul(a, bt.T.copy()))


def test_topk_topp_worked_example():
    probs = np.array([0.4, 0.3, 0.2, 0.1])
    out = O.probs_from_logits(np.log(probs), temperature=1.0, top_k=2, top_p=0.5)
    assert out.tolist() == [1.0, 0.0, 0.0, 0.0]
    out = O.probs_from_logits(np.log(probs), temperature=1.0, top_k=2, top_p=1.0)
    assert np.allclose(out, [0.4 / 0.7, 0.3 / 0.7, 0, 0])


def test_greedy_is_first_index_of_strict_max():
    assert O.argmax(np.array([1.0, 3.0, 3.0, 2.0])) == 1
    assert O.argmax(np.array([-np.inf, -np.inf])) == 0
    assert O.probs_from_logits(np.array([0.0, 5.0, 5.0]), temperature=0.0).tolist() == [0, 1, 0]


def test_sample_from_distribution_inverse_cdf():
    # One NextFloat draw walked in natural index order (Distribution.ts:93-104).
    st = 9
    r = O.Rng(st)
    u = r.next_float()
    probs = np.array([0.0, 0.25, 0.0, 0.5, 0.25])
    idx, st2 = O.sample_from_logits(np.log(np.where(probs > 0, probs, 1e-300)), st, temperature=1.0, top_k=0, top_p=0.999999)
    cdf = np.cumsum(probs)
    assert st2 == r.state[0]
    assert idx == int(np.searchsorted(cdf, u, side="left"))


SHAPES_F64 = [(256, 128, 512), (7, 5, 3), (13, 128, 9), (16, 13, 5), (1, 1, 1)]  # Compute.Test.ts:130-136
SHAPES_NT = [(33, 70, 19), (7, 5, 3), (1, 1, 1)]  # Compute.Test.ts:280, FfiGuard.Test.ts:168


def _ref():
    r = O.ref_lib()
    if r is None:
        pytest.skip("oracle/_ref not built (reference tree absent on this machine)")
    return r


def _p(a, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


@pytest.mark.parametrize("m,k,n", SHAPES_F64)
def test_oracle_matmul_agrees_with_reference_c_kernels_f64(m, k, n):
    R = _ref()
    rng = np.random.default_rng(9)
    a = rng.standard_normal((m, k))
    b = rng.standard_normal((k, n))
    got = np.empty((m, n))
    R.RefMatMulF64(_p(a, ctypes.c_double), _p(b, ctypes.c_double), _p(got, ctypes.c_double), m, k, n, 8)
    want = O.matmul(a, b)
    assert np.max(np.abs(want - got) / (np.abs(want) + 1e-9)) < 1e-10


@pytest.mark.parametrize("m,k,n", SHAPES_NT)
def test_oracle_matmul_nt_tn_agree_with_reference_c_kernels(m, k, n):
    R = _ref()
    rng = np.random.default_rng(31)
    a = rng.standard_normal((m, k))
    bt = rng.standard_normal((n, k))
    dout = rng.standard_normal((m, n))
    seed = rng.standard_normal((m, n))
    dbseed = rng.standard_normal((k, n))

    def scaled(got, want):
        return np.max(np.abs(want - got) / np.maximum(np.abs(want), 1))

    for dt, ct, tol, nt, tn in ((np.float64, ctypes.c_double, 1e-10, R.RefMatMulNTF64, R.RefMatMulTNF64),
                                (np.float32, ctypes.c_float, 1e-4, R.RefMatMulNTF32, R.RefMatMulTNF32)):
        A, BT, D = a.astype(dt), bt.astype(dt), dout.astype(dt)
        want = O.matmul_nt(A.astype(np.float64), BT.astype(np.float64))
        out = np.full((m, n), 7, dtype=dt)
        nt(_p(A, ct), _p(BT, ct), _p(out, ct), m, k, n, 0, 8)
        assert scaled(out, want) < tol
        acc = seed.astype(dt).copy()
        nt(_p(A, ct), _p(BT, ct), _p(acc, ct), m, k, n, 1, 8)
        assert scaled(acc, want + seed.astype(dt).astype(np.float64)) < tol
        db = dbseed.astype(dt).copy()
        tn(_p(A, ct), _p(D, ct), _p(db, ct), m, k, n, 1)
        want_tn = O.matmul_tn(A.astype(np.float64), D.astype(np.float64), dbseed.astype(dt).astype(np.float64).copy(), acc=True)
        assert scaled(db, want_tn) < tol


def test_committed_golden_vectors_still_match():
    """tests/golden/oracle_golden.npz pins the oracle's outputs (made by tests/golden/make_golden.py)."""
    path = os.path.join(GOLDEN, "oracle_golden.npz")
    if not os.path.exists(path):
        pytest.skip("golden fixture not generated")
    from tests.golden.make_golden import compute_goldens
    want = np.load(path)
    got = compute_goldens()
    for key in want.files:
        if want[key].dtype.kind in "iu":
            assert np.array_equal(want[key], got[key]), key
        else:
            assert np.allclose(want[key], got[key], rtol=0, atol=1e-12), key
