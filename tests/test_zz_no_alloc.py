"""ShahdMatMulNTF32NoAlloc against MatMulNTF32, both through the C ABI.

The entry point stages operands in a fixed per-device array instead of a cudaMalloc'd workspace. It must
give MatMulNTF32's results (same kernel; the seam's f32 tolerance, Tests/FfiGuard.Test.ts:146-200, is
1e-4 scaled error) on consecutive calls that reuse the array, refuse calls beyond its limit with a
clear error, and leave the device's free memory unchanged. Collected last so it also runs after every
other GPU test in the same process.
"""
import ctypes

import numpy as np
import pytest

from tests.helpers import O, pkg

pytestmark = pytest.mark.gpu

TOL = 1e-4
LIMIT = 16 << 20


def _fp(x):
    return x.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _noalloc(lib, a, bt, out, m, k, n, acc):
    return lib.ShahdMatMulNTF32NoAlloc(_fp(a), _fp(bt), _fp(out), m, k, n, acc)


def _existing(lib, a, bt, out, m, k, n, acc):
    lib.MatMulNTF32(_fp(a), _fp(bt), _fp(out), m, k, n, acc)
    assert lib.ShahdLastError() == b""


def _scaled(got, want):
    return float(np.max(np.abs(want.astype(np.float64) - got) / np.maximum(np.abs(want), 1)))


def _case(rng, m, k, n):
    a = rng.standard_normal((m, k)).astype(np.float32)
    bt = rng.standard_normal((n, k)).astype(np.float32)
    seed = rng.standard_normal((m, n)).astype(np.float32)
    return a, bt, seed


def test_two_calls_in_a_row_match_matmul_nt_f32():
    lib = pkg.load()
    rng = np.random.default_rng(31)
    # consecutive calls of different shapes reuse the same array; the second one is larger, so the
    # first call's operands sit where the second call's B and C now start
    for (m, k, n), acc in (((33, 70, 19), 0), ((300, 256, 513), 1)):
        a, bt, seed = _case(rng, m, k, n)
        want = seed.copy()
        _existing(lib, a, bt, want, m, k, n, acc)
        got = seed.copy()
        assert _noalloc(lib, a, bt, got, m, k, n, acc) == pkg._lib.SHAHD_OK, lib.ShahdLastError()
        assert _scaled(got, want) < TOL
        ref = O.matmul_nt(a.astype(np.float64), bt.astype(np.float64)) + (seed if acc else 0)
        assert _scaled(got, ref) < TOL


def test_known_answer_and_limit():
    lib = pkg.load()
    a = np.array([1, 2, 3, 4, 5, 6], np.float32)
    bt = np.array([1, 0, -1, 2, 1, 0], np.float32)
    out = np.full(4, 7, np.float32)
    assert _noalloc(lib, a, bt, out, 2, 3, 2, 0) == pkg._lib.SHAHD_OK
    assert out.tolist() == [-2, 4, -2, 13]  # Tests/MatMulNT.Test.ts:43-52
    # 1024x1024 operands: 12 MiB of the 16 MiB fits; 2048x1024x1024 does not
    m = k = n = 1024
    assert 4 * (m * k + n * k + m * n) <= LIMIT
    big = np.zeros(2048 * 1024, np.float32)
    out = np.full(2048 * 1024, 3, np.float32)
    rc = _noalloc(lib, big, big[: 1024 * 1024], out, 2048, 1024, 1024, 0)
    assert rc == pkg._lib.SHAHD_EINVAL
    msg = lib.ShahdLastError().decode()
    assert "limit" in msg and str(LIMIT) in msg
    assert np.all(out == 3)  # refused before touching anything
    assert _noalloc(lib, a, bt, out[:4], 0, 3, 2, 0) == pkg._lib.SHAHD_EINVAL


def _cudart():
    """The CUDA runtime library of the toolkit (cudaMemGetInfo), without importing torch."""
    import ctypes.util
    import glob
    import os

    cands = [ctypes.util.find_library("cudart")]
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cands += sorted(glob.glob(os.path.join(home, "lib64", "libcudart.so*")))
    for c in cands:
        if c:
            try:
                return ctypes.CDLL(c)
            except OSError:
                continue
    pytest.fail("no CUDA runtime library found for cudaMemGetInfo")


def _free_bytes(rt) -> int:
    free, total = ctypes.c_size_t(), ctypes.c_size_t()
    assert rt.cudaDeviceSynchronize() == 0
    assert rt.cudaMemGetInfo(ctypes.byref(free), ctypes.byref(total)) == 0
    return free.value


def test_free_device_memory_unchanged():
    # the entry point's whole promise: no cudaMalloc/cudaFree, however large the calls get (up to the limit)
    rt = _cudart()
    lib = pkg.load()
    rng = np.random.default_rng(5)
    a, bt, seed = _case(rng, 64, 64, 64)
    out = seed.copy()
    assert _noalloc(lib, a, bt, out, 64, 64, 64, 0) == pkg._lib.SHAHD_OK  # set-up done by now
    free0 = _free_bytes(rt)
    for m, k, n in ((1024, 1024, 1024), (5, 900, 777), (64, 64, 64)):
        a, bt, seed = _case(rng, m, k, n)
        out = seed.copy()
        assert _noalloc(lib, a, bt, out, m, k, n, 1) == pkg._lib.SHAHD_OK, lib.ShahdLastError()
        assert _free_bytes(rt) == free0, (m, k, n)
