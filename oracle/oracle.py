"""ctypes wrapper of the CPU oracle (oracle/liboracle.so) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs import this
module, and only as the checker or the timed CPU baseline. The shipped library never loads it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_matmul.so")

_i32 = ctypes.c_int32
_dp = ctypes.POINTER(ctypes.c_double)
_ip = ctypes.POINTER(ctypes.c_int32)
_up = ctypes.POINTER(ctypes.c_uint32)


class OracleCfg(ctypes.Structure):
    _fields_ = [
        ("embed_dim", _i32), ("num_layers", _i32), ("num_heads", _i32), ("kv_heads", _i32),
        ("block_size", _i32), ("vocab_size", _i32), ("mlp_hidden", _i32), ("position_scheme", _i32),
        ("norm_kind", _i32), ("mlp_kind", _i32), ("weight_tying", _i32), ("use_scaled_residual_init", _i32),
        ("precision_f32", _i32), ("pad_", _i32), ("layer_norm_eps", ctypes.c_double), ("init_scale", ctypes.c_double),
    ]


class OracleSampling(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_double), ("top_k", _i32), ("pad_", _i32), ("top_p", ctypes.c_double)]


@dataclass(frozen=True)
class Shape:
    """Model knobs (Brain/Config/Constants.ts:11-26) with MlpHidden resolved."""

    embed_dim: int
    num_layers: int
    num_heads: int
    block_size: int
    vocab_size: int
    mlp_hidden: int
    kv_heads: int | None = None
    position_scheme: str = "Learned"
    norm_kind: str = "LayerNorm"
    mlp_kind: str = "Relu"
    weight_tying: bool = True
    use_scaled_residual_init: bool = True
    precision: str = "F64"
    layer_norm_eps: float = 1e-5
    init_scale: float = 0.02

    def ctypes_cfg(self) -> OracleCfg:
        return OracleCfg(
            self.embed_dim, self.num_layers, self.num_heads, self.kv_heads or self.num_heads, self.block_size,
            self.vocab_size, self.mlp_hidden, {"Learned": 0, "Rope": 1}[self.position_scheme],
            {"LayerNorm": 0, "RmsNorm": 1}[self.norm_kind], {"Relu": 0, "SwiGlu": 1, "GeGlu": 2}[self.mlp_kind],
            int(self.weight_tying), int(self.use_scaled_residual_init), int(self.precision == "F32"), 0,
            self.layer_norm_eps, self.init_scale,
        )


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when REF_ROOT names a reference checkout)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(os.path.join(HERE, f)) > t for f in ("oracle.c", "oracle.h"))


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if _stale():
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_mix_seed.restype = ctypes.c_uint32
        L.oracle_mix_seed.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        L.oracle_rng_next_u32.restype = ctypes.c_uint32
        L.oracle_rng_next_u32.argtypes = [_up]
        L.oracle_rng_next_float.restype = ctypes.c_double
        L.oracle_rng_next_float.argtypes = [_up]
        L.oracle_rng_next_gaussian.restype = ctypes.c_double
        L.oracle_rng_next_gaussian.argtypes = [_up]
        L.oracle_create_streams.argtypes = [ctypes.c_uint32, _up]
        L.oracle_param_count.restype = ctypes.c_int64
        L.oracle_param_count.argtypes = [ctypes.POINTER(OracleCfg)]
        L.oracle_init_params.argtypes = [ctypes.POINTER(OracleCfg), ctypes.c_uint32, _dp]
        for name in ("oracle_matmul",):
            getattr(L, name).argtypes = [_dp, _dp, _dp, _i32, _i32, _i32]
        for name in ("oracle_matmul_nt", "oracle_matmul_tn"):
            getattr(L, name).argtypes = [_dp, _dp, _dp, _i32, _i32, _i32, _i32]
        L.oracle_model_create.restype = ctypes.c_void_p
        L.oracle_model_create.argtypes = [ctypes.POINTER(OracleCfg), _dp]
        L.oracle_model_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_cache_create.restype = ctypes.c_void_p
        L.oracle_cache_create.argtypes = [ctypes.c_void_p]
        L.oracle_cache_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_cache_length.argtypes = [ctypes.c_void_p]
        L.oracle_cache_read.argtypes = [ctypes.c_void_p, _i32, _i32, _dp, _dp]
        L.oracle_cached_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _i32, _i32, _dp]
        L.oracle_prefill.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _ip, _i32]
        L.oracle_forward.argtypes = [ctypes.c_void_p, _ip, _i32, _dp]
        L.oracle_forward_last_logits.argtypes = [ctypes.c_void_p, _ip, _i32, _dp]
        L.oracle_argmax.argtypes = [_dp, _i32]
        L.oracle_probs_from_logits.argtypes = [_dp, _i32, ctypes.POINTER(OracleSampling), _dp]
        L.oracle_sample_from_distribution.argtypes = [_dp, _i32, _up]
        L.oracle_sample_from_logits.argtypes = [_dp, _i32, ctypes.POINTER(OracleSampling), _up]
        for name in ("oracle_cached_generate", "oracle_generate"):
            getattr(L, name).argtypes = [ctypes.c_void_p, _ip, _i32, _i32, ctypes.POINTER(OracleSampling), _up, _ip]
        L.oracle_cached_generate_batch.argtypes = [
            ctypes.c_void_p, _ip, _i32, _i32, _i32, ctypes.POINTER(OracleSampling), _up, _ip, _i32]
        L.oracle_decoder_create.restype = ctypes.c_void_p
        L.oracle_decoder_create.argtypes = [ctypes.c_void_p, _ip, _i32]
        L.oracle_decoder_push.argtypes = [ctypes.c_void_p, _i32]
        L.oracle_decoder_logits.restype = _dp
        L.oracle_decoder_logits.argtypes = [ctypes.c_void_p]
        L.oracle_decoder_cache_length.argtypes = [ctypes.c_void_p]
        L.oracle_decoder_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_set_threads.argtypes = [_i32]
        L.oracle_speculative_round.argtypes = [_dp, _dp, _ip, _i32, _i32, _i32, ctypes.POINTER(OracleSampling), _up,
                                               _ip, ctypes.POINTER(ctypes.c_int)]
        L.oracle_speculative_sample.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _ip, _i32, _i32,
                                                ctypes.POINTER(OracleSampling), _up, _i32, _ip, _ip]
        L.oracle_check_trajectories.argtypes = [ctypes.c_void_p, _ip, _i32, _i32, _ip, _i32, ctypes.c_double, _i32,
                                                _ip, _ip, _ip, _dp]
        L.oracle_fused_attention.argtypes = [_dp, _dp, _dp, _i32, _i32, _i32, _i32, ctypes.c_double, _dp]
        L.oracle_last_error.restype = ctypes.c_char_p
        _LIB = L
    return _LIB


class OracleError(RuntimeError):
    pass


def _check(rc: int) -> None:
    if rc != 0:
        raise OracleError(lib().oracle_last_error().decode())


def _d(a: np.ndarray):
    assert a.dtype == np.float64 and a.flags.c_contiguous
    return a.ctypes.data_as(_dp)


def _i(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_ip)


def _u(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(_up)


def sampling(temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0) -> OracleSampling:
    return OracleSampling(temperature, top_k, 0, top_p)


GREEDY = dict(temperature=0.0, top_k=0, top_p=1.0)


# ---- RNG --------------------------------------------------------------------------------------

class Rng:
    """SeededRng (Brain/Random/SeededRng.ts:14-48)."""

    def __init__(self, seed: int):
        self.state = np.array([seed & 0xFFFFFFFF], dtype=np.uint32)

    def next_u32(self) -> int:
        return int(lib().oracle_rng_next_u32(_u(self.state)))

    def next_float(self) -> float:
        return float(lib().oracle_rng_next_float(_u(self.state)))

    def next_gaussian(self) -> float:
        return float(lib().oracle_rng_next_gaussian(_u(self.state)))


def mix_seed(seed: int, stream: int) -> int:
    return int(lib().oracle_mix_seed(seed & 0xFFFFFFFF, stream))


def create_streams(seed: int) -> list[int]:
    out = np.zeros(4, dtype=np.uint32)
    lib().oracle_create_streams(seed & 0xFFFFFFFF, _u(out))
    return [int(v) for v in out]


def set_threads(n: int) -> None:
    """Threads of the oracle's batched matmuls (prefill and full forward); results do not depend on it."""
    lib().oracle_set_threads(int(n))


def uniform_ids(count: int, vocab: int, seed: int) -> np.ndarray:
    """Token ids floor(NextFloat() * vocab) from SeededRng(seed), as Scripts/Bench.ts:41-42 draws them."""
    r = Rng(seed)
    return np.array([int(r.next_float() * vocab) for _ in range(count)], dtype=np.int32)


# ---- parameters -------------------------------------------------------------------------------

def param_count(shape: Shape) -> int:
    cfg = shape.ctypes_cfg()
    n = lib().oracle_param_count(ctypes.byref(cfg))
    if n < 0:
        raise OracleError(lib().oracle_last_error().decode())
    return int(n)


def init_params(shape: Shape, seed: int) -> np.ndarray:
    """Flat f64 parameters in Shahd.Parameters() order, drawn as the reference constructor draws them."""
    cfg = shape.ctypes_cfg()
    p = np.empty(param_count(shape), dtype=np.float64)
    _check(lib().oracle_init_params(ctypes.byref(cfg), seed & 0xFFFFFFFF, _d(p)))
    return p


# ---- matmul semantics -------------------------------------------------------------------------

def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), dtype=np.float64)
    lib().oracle_matmul(_d(np.ascontiguousarray(a, np.float64)), _d(np.ascontiguousarray(b, np.float64)), _d(out), m, k, n)
    return out


def matmul_nt(a: np.ndarray, bt: np.ndarray, out: np.ndarray | None = None, acc: bool = False) -> np.ndarray:
    m, k = a.shape
    n = bt.shape[0]
    if out is None:
        out = np.zeros((m, n), dtype=np.float64)
    lib().oracle_matmul_nt(_d(np.ascontiguousarray(a, np.float64)), _d(np.ascontiguousarray(bt, np.float64)), _d(out),
                           m, k, n, int(acc))
    return out


def matmul_tn(a: np.ndarray, dout: np.ndarray, db: np.ndarray | None = None, acc: bool = False) -> np.ndarray:
    m, k = a.shape
    n = dout.shape[1]
    if db is None:
        db = np.zeros((k, n), dtype=np.float64)
    lib().oracle_matmul_tn(_d(np.ascontiguousarray(a, np.float64)), _d(np.ascontiguousarray(dout, np.float64)), _d(db),
                           m, k, n, int(acc))
    return db


# ---- model ------------------------------------------------------------------------------------

class Model:
    """The reference model (Brain/Nn/Shahd.ts) with its cached and uncached forwards."""

    def __init__(self, shape: Shape, params: np.ndarray):
        self.shape = shape
        self.cfg = shape.ctypes_cfg()
        self.params = np.ascontiguousarray(params, dtype=np.float64)
        if self.params.size != param_count(shape):
            raise ValueError(f"expected {param_count(shape)} parameters, got {self.params.size}")
        self.handle = lib().oracle_model_create(ctypes.byref(self.cfg), _d(self.params))
        if not self.handle:
            raise OracleError(lib().oracle_last_error().decode())
        self.vocab = shape.vocab_size

    def __del__(self):
        if getattr(self, "handle", None):
            lib().oracle_model_destroy(self.handle)
            self.handle = None

    def new_cache(self) -> "Cache":
        return Cache(self)

    def forward(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.vocab), dtype=np.float64)
        _check(lib().oracle_forward(self.handle, _i(ids), ids.size, _d(out)))
        return out

    def forward_last_logits(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.vocab, dtype=np.float64)
        _check(lib().oracle_forward_last_logits(self.handle, _i(ids), ids.size, _d(out)))
        return out

    def cached_generate(self, prompt, max_new: int, temperature=0.0, top_k=0, top_p=1.0, rng_state: int = 1):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(prompt.size + max(max_new, 0), dtype=np.int32)
        st = np.array([rng_state & 0xFFFFFFFF], dtype=np.uint32)
        o = sampling(temperature, top_k, top_p)
        _check(lib().oracle_cached_generate(self.handle, _i(prompt), prompt.size, max_new, ctypes.byref(o), _u(st), _i(out)))
        return out, int(st[0])

    def generate(self, prompt, max_new: int, temperature=0.0, top_k=0, top_p=1.0, rng_state: int = 1):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(prompt.size + max(max_new, 0), dtype=np.int32)
        st = np.array([rng_state & 0xFFFFFFFF], dtype=np.uint32)
        o = sampling(temperature, top_k, top_p)
        _check(lib().oracle_generate(self.handle, _i(prompt), prompt.size, max_new, ctypes.byref(o), _u(st), _i(out)))
        return out, int(st[0])

    def check_trajectories(self, prompts: np.ndarray, ids: np.ndarray, tol: float, threads: int = 0) -> dict:
        """Teacher-forced judgement of greedy ids [nseq, nnew] produced elsewhere from prompts [nseq, plen]:
        each id must be the oracle's argmax on the same prefix unless the oracle's top-2 margin is within
        tol x logit range. Returns per-sequence failing steps, first failing step (-1 none), near ties
        met with a different id and the largest (max - chosen) logit gap relative to the range."""
        prompts = np.ascontiguousarray(prompts, dtype=np.int32)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        nseq, plen = prompts.shape
        nnew = ids.shape[1]
        fails = np.zeros(nseq, np.int32)
        first = np.full(nseq, -1, np.int32)
        ties = np.zeros(nseq, np.int32)
        gap = np.zeros(nseq, np.float64)
        threads = threads or (os.cpu_count() or 1)
        _check(lib().oracle_check_trajectories(self.handle, _i(prompts), nseq, plen, _i(ids), nnew, float(tol), threads,
                                               _i(fails), _i(first), _i(ties), _d(gap)))
        return {"fails": fails, "first_fail": first, "near_ties": ties, "max_gap": gap}

    def cached_generate_batch(self, prompts: np.ndarray, max_new: int, rng_states: np.ndarray | None = None,
                              threads: int = 1, temperature=0.0, top_k=0, top_p=1.0) -> np.ndarray:
        prompts = np.ascontiguousarray(prompts, dtype=np.int32)
        nseq, plen = prompts.shape
        out = np.empty((nseq, plen + max_new), dtype=np.int32)
        st = np.ones(nseq, dtype=np.uint32) if rng_states is None else np.ascontiguousarray(rng_states, np.uint32).copy()
        o = sampling(temperature, top_k, top_p)
        _check(lib().oracle_cached_generate_batch(self.handle, _i(prompts), nseq, plen, max_new, ctypes.byref(o), _u(st),
                                                  _i(out), threads))
        return out


class Cache:
    """KvCache (Brain/Sampling/KvCache.ts) bound to one model."""

    def __init__(self, model: Model):
        self.model = model
        self.handle = lib().oracle_cache_create(model.handle)

    def __del__(self):
        if getattr(self, "handle", None):
            lib().oracle_cache_destroy(self.handle)
            self.handle = None

    @property
    def length(self) -> int:
        return int(lib().oracle_cache_length(self.handle))

    def step(self, token: int, position: int | None = None) -> np.ndarray:
        """CachedForwardStep: logits for the token after `token`, appending its K/V."""
        if position is None:
            position = self.length
        out = np.empty(self.model.vocab, dtype=np.float64)
        _check(lib().oracle_cached_step(self.model.handle, self.handle, int(token), int(position), _d(out)))
        return out

    def prefill(self, ids) -> None:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        _check(lib().oracle_prefill(self.model.handle, self.handle, _i(ids), ids.size))

    def read(self, layer: int, kv_head: int) -> tuple[np.ndarray, np.ndarray]:
        s = self.model.shape
        d = s.embed_dim // s.num_heads
        cap = s.block_size
        k = np.empty(cap * d, dtype=np.float64)
        v = np.empty(cap * d, dtype=np.float64)
        n = lib().oracle_cache_read(self.handle, layer, kv_head, _d(k), _d(v))
        if n < 0:
            raise OracleError(lib().oracle_last_error().decode())
        return k[: n * d].reshape(n, d), v[: n * d].reshape(n, d)


class Decoder:
    """CachedDecoder (Brain/Sampling/CachedForward.ts:113-150)."""

    def __init__(self, model: Model, prompt):
        self.model = model
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        self.handle = lib().oracle_decoder_create(model.handle, _i(prompt), prompt.size)
        if not self.handle:
            raise OracleError(lib().oracle_last_error().decode())

    def __del__(self):
        if getattr(self, "handle", None):
            lib().oracle_decoder_destroy(self.handle)
            self.handle = None

    @property
    def logits(self) -> np.ndarray:
        p = lib().oracle_decoder_logits(self.handle)
        return np.ctypeslib.as_array(p, shape=(self.model.vocab,)).copy()

    @property
    def cache_length(self) -> int:
        return int(lib().oracle_decoder_cache_length(self.handle))

    def push(self, token: int) -> None:
        _check(lib().oracle_decoder_push(self.handle, int(token)))


# ---- sampling ---------------------------------------------------------------------------------

def argmax(logits) -> int:
    lg = np.ascontiguousarray(logits, dtype=np.float64)
    return int(lib().oracle_argmax(_d(lg), lg.size))


def probs_from_logits(logits, temperature: float, top_k: int = 0, top_p: float = 1.0) -> np.ndarray:
    lg = np.ascontiguousarray(logits, dtype=np.float64)
    out = np.empty_like(lg)
    o = sampling(temperature, top_k, top_p)
    lib().oracle_probs_from_logits(_d(lg), lg.size, ctypes.byref(o), _d(out))
    return out


def sample_from_logits(logits, rng_state: int, temperature: float, top_k: int = 0, top_p: float = 1.0):
    lg = np.ascontiguousarray(logits, dtype=np.float64)
    st = np.array([rng_state & 0xFFFFFFFF], dtype=np.uint32)
    o = sampling(temperature, top_k, top_p)
    idx = lib().oracle_sample_from_logits(_d(lg), lg.size, ctypes.byref(o), _u(st))
    return int(idx), int(st[0])


def speculative_round(target_logits, draft_logits, proposals, budget: int, rng_state: int, temperature: float,
                      top_k: int = 0, top_p: float = 1.0):
    """One SpeculativeSample verification round on given logits (target [g+1, V], draft [g, V]):
    returns (ids appended, accepted proposals, the Rng state after the round)."""
    t = np.ascontiguousarray(target_logits, dtype=np.float64)
    d = np.ascontiguousarray(draft_logits, dtype=np.float64)
    prop = np.ascontiguousarray(proposals, dtype=np.int32)
    g, V = prop.size, t.shape[-1]
    out = np.zeros(g + 1, dtype=np.int32)
    st = np.array([rng_state & 0xFFFFFFFF], dtype=np.uint32)
    acc = ctypes.c_int()
    o = sampling(temperature, top_k, top_p)
    n = lib().oracle_speculative_round(_d(t), _d(d), _i(prop), g, V, budget, ctypes.byref(o), _u(st), _i(out),
                                       ctypes.byref(acc))
    return out[:n].tolist(), int(acc.value), int(st[0])


def speculative_sample(target: "Model", draft: "Model", prompt, max_new: int, rng_state: int, temperature: float,
                       top_k: int = 0, top_p: float = 1.0, gamma: int = 4):
    """SpeculativeSample (Brain/Reasoning/SpeculativeSampling.ts:38-115): ids, Rng state, [calls, drafted,
    accepted]."""
    prompt = np.ascontiguousarray(prompt, dtype=np.int32)
    out = np.zeros(prompt.size + max_new, dtype=np.int32)
    st = np.array([rng_state & 0xFFFFFFFF], dtype=np.uint32)
    stats = np.zeros(3, dtype=np.int32)
    o = sampling(temperature, top_k, top_p)
    _check(lib().oracle_speculative_sample(target.handle, draft.handle, _i(prompt), prompt.size, max_new,
                                           ctypes.byref(o), _u(st), gamma, _i(out), _i(stats)))
    return out.tolist(), int(st[0]), stats.tolist()


# ---- reference C kernels (oracle/_ref) --------------------------------------------------------

_REF = None


def fused_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, rope_base: float = 10000.0) -> np.ndarray:
    """FusedAttention of one sequence (MultiHeadAttention.ts:46-74 core: RoPE on Q and K, CausalSoftmax,
    @ V; GQA head h reads kv head h / (H / Hk)); q [T, H, d], k and v [T, Hk, d] -> [T, H, d], f64. Row p
    is also a decode step's AttendRow (CachedRowMath.ts:60-86) over rows 0..p."""
    q = np.ascontiguousarray(q, dtype=np.float64)
    k = np.ascontiguousarray(k, dtype=np.float64)
    v = np.ascontiguousarray(v, dtype=np.float64)
    T, H, d = q.shape
    Hk = k.shape[1]
    out = np.empty((T, H, d), dtype=np.float64)
    _check(lib().oracle_fused_attention(_d(q), _d(k), _d(v), T, H, Hk, d, float(rope_base), _d(out)))
    return out


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own C matmul kernels behind a pthread fan-out, or None when not built."""
    global _REF
    if _REF is None and os.path.exists(REF_LIB_PATH):
        R = ctypes.CDLL(REF_LIB_PATH)
        fp = ctypes.POINTER(ctypes.c_float)
        R.RefMatMulNTF32.argtypes = [fp, fp, fp, _i32, _i32, _i32, _i32, _i32]
        R.RefMatMulNTF64.argtypes = [_dp, _dp, _dp, _i32, _i32, _i32, _i32, _i32]
        R.RefMatMulF32.argtypes = [fp, fp, fp, _i32, _i32, _i32, _i32]
        R.RefMatMulF64.argtypes = [_dp, _dp, _dp, _i32, _i32, _i32, _i32]
        R.RefMatMulTNF32.argtypes = [fp, fp, fp, _i32, _i32, _i32, _i32]
        R.RefMatMulTNF64.argtypes = [_dp, _dp, _dp, _i32, _i32, _i32, _i32]
        _REF = R
    return _REF
