"""CPU checks of the C-ABI library: it loads, exports every symbol include/shahd_b200.h declares, and its
host logic (parameter layout, the reference's weight init, argument validation) is right without a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

from tests.helpers import ARCHS, O, oracle_shape, pkg

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "shahd_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", text, flags=re.M)
    return sorted({n for n in names if n not in ("if", "while", "for", "return", "sizeof")})


def test_library_loads_and_exports_every_declared_symbol():
    lib = pkg.load()
    names = declared_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), f"libshahd_b200.so does not export {n}"
    assert set(names) == set(pkg._lib.SIGNATURES), "ctypes table and header disagree"


def test_go_ffi_symbol_set_is_complete():
    # GoFfiBackend.ts:92-151 loads exactly these names
    lib = pkg.load()
    for n in ("MatMulF64", "MatMulNTF64", "MatMulTNF64", "MatMulF32", "MatMulNTF32", "MatMulTNF32", "SetKernelThreads",
              "ShahdCpuSupportsAvx2Fma", "SetScalarKernels"):
        assert hasattr(lib, n)


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_param_count_matches_reference_layout(label, arch):
    cfg = pkg.ModelConfig(**arch)
    assert pkg.decode.param_count(cfg) == O.param_count(oracle_shape(cfg))


@pytest.mark.parametrize("label,arch", ARCHS, ids=[a[0] for a in ARCHS])
def test_init_params_bit_exact_with_oracle(label, arch):
    cfg = pkg.ModelConfig(**arch)
    got = pkg.init_params(cfg, seed=1)
    want = O.init_params(oracle_shape(cfg, "F32"), seed=1)
    assert got.dtype == np.float32
    assert np.array_equal(got.astype(np.float64), want)


def test_init_params_baseline_shapes():
    for w in pkg.configs.WORKLOADS.values():
        n = pkg.decode.param_count(w.model)
        assert n == O.param_count(oracle_shape(w.model))
    mc = pkg.configs.MICROCHAT.model
    p = pkg.init_params(mc, seed=1)
    q = O.init_params(oracle_shape(mc, "F32"), seed=1)
    assert np.array_equal(p.astype(np.float64), q)


def test_validate_matmul_args_messages():
    # Tests/FfiGuard.Test.ts:86-109
    v = pkg.backend.validate_matmul_args
    F64 = lambda n: np.zeros(n)  # noqa: E731
    v("Test", F64(6), F64(12), F64(8), 2, 3, 4)
    with pytest.raises(ValueError, match="A has 5 elements"):
        v("Test", F64(5), F64(12), F64(8), 2, 3, 4)
    with pytest.raises(ValueError, match="B has 11 elements"):
        v("Test", F64(6), F64(11), F64(8), 2, 3, 4)
    with pytest.raises(ValueError, match="Out has 7 elements"):
        v("Test", F64(6), F64(12), F64(7), 2, 3, 4)
    with pytest.raises(TypeError, match="mixed buffer precisions"):
        v("Test", F64(6), np.zeros(12, np.float32), F64(8), 2, 3, 4)
    with pytest.raises(ValueError, match="empty"):
        v("Test", F64(0), F64(12), F64(8), 2, 3, 4)
    with pytest.raises(ValueError, match="dimension M"):
        v("Test", F64(0), F64(0), F64(0), 0, 0, 0)
    with pytest.raises(ValueError, match="dimension K"):
        v("Test", F64(6), F64(12), F64(8), 2, 1.5, 4)
    with pytest.raises(TypeError, match="Float64Array or Float32Array"):
        v("Test", [1, 2, 3, 4, 5, 6], F64(12), F64(8), 2, 3, 4)
    v("Test", F64(6), F64(8), F64(12), 2, 3, 4, "TN")
    with pytest.raises(ValueError, match="Db has 11 elements"):
        v("Test", F64(6), F64(8), F64(11), 2, 3, 4, "TN")
    with pytest.raises(ValueError, match="DOut has 7 elements"):
        v("Test", F64(6), F64(7), F64(12), 2, 3, 4, "TN")


def test_native_dim_validation_records_error_without_touching_memory():
    lib = pkg.load()
    out = np.full(4, 7.0)
    a = np.ones(4)
    p = a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))
    lib.MatMulF64(p, p, out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), 0, 2, 2)
    assert "dimension M" in pkg._lib.last_error()
    assert out.tolist() == [7.0] * 4


def test_bad_model_config_rejected_on_host():
    bad = pkg.ModelConfig(embed_dim=10, num_layers=1, num_heads=3, block_size=4, vocab_size=5, mlp_hidden=8)
    with pytest.raises(ValueError, match="divisible"):
        pkg.decode.param_count(bad)


def test_no_device_is_an_error_not_a_fallback():
    from tests.conftest import has_gpu
    if has_gpu():
        pytest.skip("a GPU is present")
    lib = pkg.load()
    assert lib.ShahdGpuAvailable() == 0
    assert lib.ShahdCpuSupportsAvx2Fma() == 0
    cfg = pkg.ModelConfig(**ARCHS[0][1])
    with pytest.raises(pkg._lib.ShahdError) as e:
        pkg.Session(cfg, pkg.init_params(cfg, 1), max_seqs=1)
    assert e.value.code == pkg._lib.SHAHD_ENODEV
    with pytest.raises(RuntimeError, match="sm_100"):
        pkg.GpuBackend()
    # the batch sampler checks its arguments, then refuses without a device
    with pytest.raises(pkg._lib.ShahdError) as e:
        pkg.sample_from_logits(np.zeros((2, 8), np.float32), pkg.GREEDY)
    assert e.value.code == pkg._lib.SHAHD_ENODEV
    with pytest.raises(pkg._lib.ShahdError, match="rng_states"):
        pkg.sample_from_logits(np.zeros((2, 8), np.float32), pkg.Sampling(1.0, 0, 1.0), None)
