"""ctypes binding of libshahd_b200.so (the C ABI declared in include/shahd_b200.h).

Loading fails loudly when the library is missing: there is no CPU path behind this package.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_vp = ctypes.c_void_p
_fp = ctypes.POINTER(ctypes.c_float)
_dp = ctypes.POINTER(ctypes.c_double)
_ip = ctypes.POINTER(ctypes.c_int32)
_up = ctypes.POINTER(ctypes.c_uint32)

SHAHD_OK = 0
SHAHD_EINVAL = -1
SHAHD_ENODEV = -2
SHAHD_ENOMEM = -3
SHAHD_ECUDA = -4
SHAHD_ESTATE = -5
SHAHD_ETIMEOUT = -6


class ShahdModelCfg(ctypes.Structure):
    _fields_ = [
        ("embed_dim", _i32), ("num_layers", _i32), ("num_heads", _i32), ("kv_heads", _i32), ("block_size", _i32),
        ("vocab_size", _i32), ("mlp_hidden", _i32), ("position_scheme", _i32), ("norm_kind", _i32),
        ("mlp_kind", _i32), ("weight_tying", _i32), ("reserved", _i32), ("layer_norm_eps", ctypes.c_double),
        ("rope_base", ctypes.c_double),
    ]


class ShahdSampling(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_double), ("top_k", _i32), ("reserved", _i32), ("top_p", ctypes.c_double)]


class ShahdSessionOpts(ctypes.Structure):
    _fields_ = [("max_seqs", _i32), ("kv_pages", _i32), ("device", _i32), ("flags", _i32)]


# name -> (restype, argtypes); every symbol include/shahd_b200.h declares
SIGNATURES = {
    "MatMulF64": (None, [_dp, _dp, _dp, _i32, _i32, _i32]),
    "MatMulNTF64": (None, [_dp, _dp, _dp, _i32, _i32, _i32, _i32]),
    "MatMulTNF64": (None, [_dp, _dp, _dp, _i32, _i32, _i32, _i32]),
    "MatMulF32": (None, [_fp, _fp, _fp, _i32, _i32, _i32]),
    "MatMulNTF32": (None, [_fp, _fp, _fp, _i32, _i32, _i32, _i32]),
    "MatMulTNF32": (None, [_fp, _fp, _fp, _i32, _i32, _i32, _i32]),
    "SetKernelThreads": (None, [ctypes.c_int]),
    "ShahdCpuSupportsAvx2Fma": (ctypes.c_int, []),
    "SetScalarKernels": (None, [ctypes.c_int]),
    "ShahdGpuAvailable": (ctypes.c_int, []),
    "ShahdLastError": (ctypes.c_char_p, []),
    "ShahdSetTensorCoreMinRows": (None, [ctypes.c_int]),
    "ShahdDeviceErrorFlag": (ctypes.c_int, []),
    "ShahdSetProgrammaticLaunch": (None, [ctypes.c_int]),
    "ShahdSetDecodeChains": (None, [ctypes.c_int]),
    "ShahdSetPersistentStep": (None, [ctypes.c_int]),
    "ShahdSetTensorCorePrefillAttention": (None, [ctypes.c_int]),
    "ShahdSetDecodeAttentionKernel": (None, [ctypes.c_int]),
    "ShahdSetFusedAttentionBlock": (None, [ctypes.c_int]),
    "ShahdSetPersistentPrefillProjections": (None, [ctypes.c_int]),
    "ShahdMatMulNTBF16Device": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    "ShahdMatMulNTF32Device": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    "ShahdMatMulNTF32NoAlloc": (ctypes.c_int, [_fp, _fp, _fp, _i32, _i32, _i32, _i32]),
    "shahd_param_count": (_i64, [ctypes.POINTER(ShahdModelCfg)]),
    "shahd_init_params": (ctypes.c_int, [ctypes.POINTER(ShahdModelCfg), _u32, _fp, _i64]),
    "shahd_session_create": (ctypes.c_int, [ctypes.POINTER(ShahdModelCfg), _vp, _i32, _i64,
                                            ctypes.POINTER(ShahdSessionOpts), ctypes.POINTER(_vp)]),
    "shahd_session_destroy": (ctypes.c_int, [_vp]),
    "shahd_reset": (ctypes.c_int, [_vp, _ip, _i32]),
    "shahd_seq_length": (_i32, [_vp, _i32]),
    "shahd_prefill": (ctypes.c_int, [_vp, _ip, _ip, _ip, _i32]),
    "shahd_step": (ctypes.c_int, [_vp, _ip, _ip, _i32, _fp, _ip]),
    "shahd_generate": (ctypes.c_int, [_vp, _ip, _ip, _i32, _i32, ctypes.POINTER(ShahdSampling), _up, _ip]),
    "shahd_generate_device": (ctypes.c_int, [_vp, _vp, _ip, _i32, _i32, ctypes.POINTER(ShahdSampling), _vp, _vp, _vp]),
    "shahd_generate_logits": (ctypes.c_int, [_vp, _ip, _ip, _i32, _i32, _ip, _fp]),
    "shahd_sync": (ctypes.c_int, [_vp]),
    "shahd_verify": (ctypes.c_int, [_vp, _ip, _ip, _ip, _i32, _fp, _ip]),
    "shahd_truncate": (ctypes.c_int, [_vp, _ip, _ip, _i32]),
    "shahd_step_launches": (_i32, [_vp, _i32]),
    "shahd_kernel_launches": (_i64, [_vp]),
    "shahd_profile": (ctypes.c_int, [_vp, _i32]),
    "shahd_profile_read": (ctypes.c_int, [_vp, _i32, _dp, ctypes.POINTER(_i64), _dp]),
    "shahd_sample_logits": (ctypes.c_int, [_fp, _i32, _i32, ctypes.POINTER(ShahdSampling), _up, _ip]),
    "shahd_speculative_round": (ctypes.c_int, [_fp, _fp, _ip, _ip, _ip, _i32, _i32, _i32, ctypes.POINTER(ShahdSampling),
                                                _up, _ip, _ip, _ip]),
    "shahd_attention_create": (ctypes.c_int, [_i32, _i32, _i32, _i32, _i32, ctypes.c_double, _i32,
                                               ctypes.POINTER(_vp)]),
    "shahd_attention_destroy": (ctypes.c_int, [_vp]),
    "shahd_attention_length": (_i32, [_vp, _i32]),
    "shahd_attention_prefill": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i32, _i32, _vp, _vp]),
    "shahd_attention_decode": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i32, _vp, _vp]),
    "shahd_last_error": (ctypes.c_char_p, []),
}

_LIB: ctypes.CDLL | None = None


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """The process-lifetime handle of libshahd_b200.so (never closed, like GoFfiBackend.ts:36-42)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(_build.SO_PATH):
        if not build_if_missing:
            raise OSError(f"libshahd_b200.so not built at {_build.SO_PATH}")
        _build.build()
    lib = ctypes.CDLL(_build.SO_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


class ShahdError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def check(rc: int) -> None:
    if rc != SHAHD_OK:
        raise ShahdError(rc, load().shahd_last_error().decode(errors="replace"))


def last_error() -> str:
    return load().ShahdLastError().decode(errors="replace")
