"""GpuBackend: the ComputeBackend seam (Brain/ComputeBackend/ComputeBackend.ts:23-42) over
libshahd_b200, shaped like GoFfiBackend (Brain/ComputeBackend/GoFfiBackend.ts:176-246).

Buffers are numpy float64/float32 arrays (the Float64Array/Float32Array of the reference); every
entry point validates with the rules and messages of ValidateMatMulArgs
(Brain/ComputeBackend/MatMulArgs.ts:45-76) before a pointer reaches the library.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

MAX_KERNEL_DIM = 2147483647


def _describe(buf) -> str:
    if buf is None:
        return "None"
    if isinstance(buf, np.ndarray):
        return {np.dtype(np.float64): "Float64Array", np.dtype(np.float32): "Float32Array"}.get(buf.dtype, f"ndarray[{buf.dtype}]")
    return type(buf).__name__


def _assert_dim(op: str, name: str, value) -> None:
    if not isinstance(value, (int, np.integer)) or isinstance(value, bool) or value < 1 or value > MAX_KERNEL_DIM:
        raise ValueError(f"{op}: dimension {name} must be an integer in [1, {MAX_KERNEL_DIM}], got {value}")


def _assert_buffer(op: str, name: str, buf, required: int, shape: str) -> None:
    if not isinstance(buf, np.ndarray) or buf.dtype not in (np.float64, np.float32):
        raise TypeError(f"{op}: {name} must be a Float64Array or Float32Array, got {_describe(buf)}")
    if buf.size == 0:
        raise ValueError(f"{op}: {name} is empty (a native kernel cannot take a pointer to zero-length memory)")
    if buf.size < required:
        raise ValueError(f"{op}: {name} has {buf.size} elements but shape {shape} needs {required}")
    if not buf.flags.c_contiguous:
        raise ValueError(f"{op}: {name} must be contiguous")


def validate_matmul_args(op: str, a, b, out, m, k, n, layout: str = "NN") -> None:
    """ValidateMatMulArgs (MatMulArgs.ts:45-76)."""
    _assert_dim(op, "M", m)
    _assert_dim(op, "K", k)
    _assert_dim(op, "N", n)
    if layout == "NN":
        bname, bsize, bshape = "B", k * n, f"[K={k},N={n}]"
    elif layout == "NT":
        bname, bsize, bshape = "Bt", n * k, f"[N={n},K={k}]"
    else:
        bname, bsize, bshape = "DOut", m * n, f"[M={m},N={n}]"
    oname, osize, oshape = ("Db", k * n, f"[K={k},N={n}]") if layout == "TN" else ("Out", m * n, f"[M={m},N={n}]")
    _assert_buffer(op, "A", a, m * k, f"[M={m},K={k}]")
    _assert_buffer(op, bname, b, bsize, bshape)
    _assert_buffer(op, oname, out, osize, oshape)
    if not (a.dtype == b.dtype == out.dtype):
        raise TypeError(
            f"{op}: mixed buffer precisions (A={_describe(a)}, {bname}={_describe(b)}, {oname}={_describe(out)}) "
            "— all operands must share the run's storage precision")


def _ptr(buf: np.ndarray):
    ct = ctypes.c_double if buf.dtype == np.float64 else ctypes.c_float
    return buf.ctypes.data_as(ctypes.POINTER(ct))


class GpuBackend:
    """Implements MatMul, MatMulInto, MatMulNtAcc, MatMulNtInto and MatMulTnAcc on the GPU."""

    HasF32 = True

    def __init__(self):
        self._lib = _lib.load()
        if not self._lib.ShahdGpuAvailable():
            raise RuntimeError("GpuBackend: no usable sm_100 (B200) device")

    @property
    def CpuSupportsAvx2Fma(self) -> bool:  # the probe name the reference selector reads
        return bool(self._lib.ShahdCpuSupportsAvx2Fma())

    def _raise_if_failed(self, op: str) -> None:
        err = _lib.last_error()
        if err:
            raise RuntimeError(err)

    def MatMul(self, A, B, M, K, N):
        out = np.empty(M * N, dtype=A.dtype if isinstance(A, np.ndarray) else np.float64)
        self.MatMulInto(A, B, out, M, K, N)
        return out

    def MatMulInto(self, A, B, Out, M, K, N) -> None:
        validate_matmul_args("GpuBackend.MatMulInto", A, B, Out, M, K, N, "NN")
        fn = self._lib.MatMulF32 if A.dtype == np.float32 else self._lib.MatMulF64
        fn(_ptr(A), _ptr(B), _ptr(Out), M, K, N)
        self._raise_if_failed("GpuBackend.MatMulInto")

    def _nt(self, A, Bt, Out, M, K, N, acc: int, op: str) -> None:
        validate_matmul_args(op, A, Bt, Out, M, K, N, "NT")
        fn = self._lib.MatMulNTF32 if A.dtype == np.float32 else self._lib.MatMulNTF64
        fn(_ptr(A), _ptr(Bt), _ptr(Out), M, K, N, acc)
        self._raise_if_failed(op)

    def MatMulNtAcc(self, A, Bt, Out, M, K, N) -> None:
        self._nt(A, Bt, Out, M, K, N, 1, "GpuBackend.MatMulNtAcc")

    def MatMulNtInto(self, A, Bt, Out, M, K, N) -> None:
        self._nt(A, Bt, Out, M, K, N, 0, "GpuBackend.MatMulNtInto")

    def MatMulTnAcc(self, A, DOut, Db, M, K, N) -> None:
        validate_matmul_args("GpuBackend.MatMulTnAcc", A, DOut, Db, M, K, N, "TN")
        fn = self._lib.MatMulTNF32 if A.dtype == np.float32 else self._lib.MatMulTNF64
        fn(_ptr(A), _ptr(DOut), _ptr(Db), M, K, N, 1)
        self._raise_if_failed("GpuBackend.MatMulTnAcc")

    def SetKernelThreads(self, n: int) -> None:
        self._lib.SetKernelThreads(int(n))

    def SetScalarKernels(self, force: bool) -> None:
        self._lib.SetScalarKernels(1 if force else 0)


def matmul_nt_bf16_device(a_ptr: int, bt_ptr: int, out_ptr: int, m: int, k: int, n: int, acc: bool = False,
                          stream: int = 0) -> None:
    """out[M,N] (+)= A[M,K] · Btᵀ with bf16 device operands and fp32 device output (tcgen05 GEMM)."""
    lib = _lib.load()
    _lib.check(lib.ShahdMatMulNTBF16Device(ctypes.c_void_p(a_ptr), ctypes.c_void_p(bt_ptr), ctypes.c_void_p(out_ptr),
                                           m, k, n, int(acc), ctypes.c_void_p(stream)))


def matmul_nt_f32_device(a_ptr: int, bt_ptr: int, out_ptr: int, m: int, k: int, n: int, acc: bool = False,
                         stream: int = 0) -> None:
    """out[M,N] (+)= A[M,K] · Btᵀ with fp32 device operands on the tensor cores (split-TF32, three passes)."""
    lib = _lib.load()
    _lib.check(lib.ShahdMatMulNTF32Device(ctypes.c_void_p(a_ptr), ctypes.c_void_p(bt_ptr), ctypes.c_void_p(out_ptr),
                                          m, k, n, int(acc), ctypes.c_void_p(stream)))
