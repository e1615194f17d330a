"""shahd-llm-stack_b200: B200 (sm_100a) backend for the Shahd KV-cached decode path.

The product is libshahd_b200.so (C ABI in include/shahd_b200.h). This package builds it, loads it with
ctypes and mirrors the reference's host-side interface over it:
  backend.GpuBackend      — the ComputeBackend seam (MatMul / MatMulInto / MatMulNtAcc / MatMulNtInto / MatMulTnAcc)
  decode.Session          — device-resident model + paged KV cache, batched cached steps, on-device generate
  decode.CachedDecoder    — CachedDecoder over one session slot
  decode.cached_generate  — CachedGenerate
  attention.FusedAttention — the attention core (RoPE, causal prefill, AttendRow decode steps) as an operator
Import with importlib (the directory name has dashes): importlib.import_module("shahd-llm-stack_b200").
"""
from . import _lib, attention, backend, build, checkpoint, configs, decode, sharding, speculative  # noqa: F401
from .attention import FusedAttention  # noqa: F401
from .backend import GpuBackend  # noqa: F401
from .decode import (  # noqa: F401
    GREEDY, CachedDecoder, ModelConfig, Sampling, Session, cached_generate, init_params, sample_from_logits)


def load():
    """Load (building if needed) libshahd_b200.so; raises when it cannot be loaded."""
    return _lib.load()
