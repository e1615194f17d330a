"""FusedAttention as an operator (the attention core of MultiHeadAttention.Forward,
Brain/Nn/MultiHeadAttention.ts:46-74, with RoPE and CausalSoftmax, then AttendRow decode steps,
Brain/Sampling/CachedRowMath.ts:60-86) over the library's device-resident paged cache.

Q/K/V and outputs are fp32 device buffers passed by address (torch CUDA tensors work: their data_ptr()).
Calls are asynchronous on `stream` (0: the operator's own stream): the buffers must stay allocated until the
stream has reached the call, so pass torch's current stream when torch owns them.
"""
from __future__ import annotations

import ctypes

from . import _lib


class FusedAttention:
    """num_heads query heads over kv_heads kv heads, head_dim 32/64/128, `capacity` positions per sequence."""

    def __init__(self, max_seqs: int, num_heads: int, kv_heads: int, head_dim: int, capacity: int,
                 rope_base: float = 10000.0, device: int = 0):
        self.lib = _lib.load()
        self.max_seqs, self.num_heads, self.kv_heads, self.head_dim = max_seqs, num_heads, kv_heads, head_dim
        self.capacity = capacity
        h = ctypes.c_void_p()
        _lib.check(self.lib.shahd_attention_create(max_seqs, num_heads, kv_heads, head_dim, capacity, float(rope_base),
                                                   device, ctypes.byref(h)))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            self.lib.shahd_attention_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def length(self, slot: int) -> int:
        return int(self.lib.shahd_attention_length(self.handle, slot))

    def prefill(self, q: int, k: int, v: int, n: int, T: int, out: int, stream: int = 0) -> None:
        """Sequences 0..n-1 restart at position 0; q [n, T, H, d], k/v [n, T, Hk, d], out [n, T, H, d]
        (device addresses, fp32)."""
        _lib.check(self.lib.shahd_attention_prefill(self.handle, q, k, v, n, T, out, stream or None))

    def decode(self, q: int, k: int, v: int, n: int, out: int, stream: int = 0) -> None:
        """One position per sequence 0..n-1: q [n, H, d], k/v [n, Hk, d] (before RoPE), out [n, H, d]."""
        _lib.check(self.lib.shahd_attention_decode(self.handle, q, k, v, n, out, stream or None))
