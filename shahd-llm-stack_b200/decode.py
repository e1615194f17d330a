"""Decode-level host API over libshahd_b200: the Brain/Sampling surface on the GPU.

  ModelConfig         Model knobs (Brain/Config/Constants.ts:11-26) + Derived (DeriveConfig.ts:8-20)
  init_params         new Shahd(Config, CreateRngStreams(seed).InitRng) as flat f32 Parameters()
  Session             device-resident model + paged KV cache over slots (one KvCache per slot)
  CachedDecoder       CachedDecoder (CachedForward.ts:113-150) bound to one slot of a Session
  cached_generate     CachedGenerate (CachedForward.ts:153-171) for one prompt
  Session.generate    CachedGenerate for a batch of independent prompts in one device loop
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _lib

_ip = ctypes.POINTER(ctypes.c_int32)
_fp = ctypes.POINTER(ctypes.c_float)
_up = ctypes.POINTER(ctypes.c_uint32)


@dataclass(frozen=True)
class ModelConfig:
    embed_dim: int
    num_layers: int
    num_heads: int
    block_size: int
    vocab_size: int
    mlp_hidden: int
    kv_heads: int | None = None
    position_scheme: str = "Learned"  # "Learned" | "Rope"
    norm_kind: str = "LayerNorm"      # "LayerNorm" | "RmsNorm"
    mlp_kind: str = "Relu"            # "Relu" | "SwiGlu" | "GeGlu"
    weight_tying: bool = True
    layer_norm_eps: float = 1e-5
    rope_base: float = 10000.0

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    @property
    def kv(self) -> int:
        return self.kv_heads or self.num_heads

    def to_c(self) -> _lib.ShahdModelCfg:
        return _lib.ShahdModelCfg(
            self.embed_dim, self.num_layers, self.num_heads, self.kv, self.block_size, self.vocab_size,
            self.mlp_hidden, {"Learned": 0, "Rope": 1}[self.position_scheme],
            {"LayerNorm": 0, "RmsNorm": 1}[self.norm_kind], {"Relu": 0, "SwiGlu": 1, "GeGlu": 2}[self.mlp_kind],
            int(self.weight_tying), 0, self.layer_norm_eps, self.rope_base)

    def matrix_params(self) -> int:
        """Parameters of the projection/MLP/head matrices read per decode step (tied head counted once)."""
        E, H, Hk, d, F, V = self.embed_dim, self.num_heads, self.kv, self.head_dim, self.mlp_hidden, self.vocab_size
        mlp = (3 if self.mlp_kind != "Relu" else 2) * E * F
        return self.num_layers * (E * H * d + 2 * E * Hk * d + H * d * E + mlp) + V * E


@dataclass(frozen=True)
class Sampling:
    """SamplingOptions (Brain/Sampling/Distribution.ts:11-15)."""

    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0

    def to_c(self) -> _lib.ShahdSampling:
        return _lib.ShahdSampling(self.temperature, self.top_k, 0, self.top_p)


GREEDY = Sampling(0.0, 0, 1.0)


def param_count(cfg: ModelConfig) -> int:
    c = cfg.to_c()
    n = _lib.load().shahd_param_count(ctypes.byref(c))
    if n < 0:
        raise ValueError(_lib.load().shahd_last_error().decode())
    return int(n)


def init_params(cfg: ModelConfig, seed: int) -> np.ndarray:
    """The reference's seeded weight init (InitScale 0.02, scaled residual init), f32 Parameters() order."""
    c = cfg.to_c()
    out = np.empty(param_count(cfg), dtype=np.float32)
    _lib.check(_lib.load().shahd_init_params(ctypes.byref(c), seed & 0xFFFFFFFF, out.ctypes.data_as(_fp), out.size))
    return out


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _pack(prompts) -> tuple[np.ndarray, np.ndarray]:
    if isinstance(prompts, np.ndarray) and prompts.ndim == 2:
        n, t = prompts.shape
        return _i32(prompts).reshape(-1), np.arange(0, (n + 1) * t, t, dtype=np.int32)
    lens = [len(p) for p in prompts]
    offs = np.zeros(len(prompts) + 1, dtype=np.int32)
    offs[1:] = np.cumsum(lens)
    flat = np.concatenate([_i32(p) for p in prompts]) if prompts else np.zeros(0, np.int32)
    return _i32(flat), offs


class Session:
    """A model resident on one GPU with `max_seqs` KV-cache slots."""

    def __init__(self, cfg: ModelConfig, params: np.ndarray, max_seqs: int, device: int = 0, kv_pages: int = 0):
        self.lib = _lib.load()
        self.cfg = cfg
        params = np.ascontiguousarray(params)
        if params.dtype not in (np.float32, np.float64):
            raise TypeError("params must be float32 or float64")
        c = cfg.to_c()
        opts = _lib.ShahdSessionOpts(max_seqs, kv_pages, device, 0)
        h = ctypes.c_void_p()
        _lib.check(self.lib.shahd_session_create(ctypes.byref(c), params.ctypes.data_as(ctypes.c_void_p),
                                                 int(params.dtype == np.float64), params.size, ctypes.byref(opts),
                                                 ctypes.byref(h)))
        self.handle = h
        self.max_seqs = max_seqs

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.shahd_session_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- KvCache surface ----
    def reset(self, slots) -> None:
        s = _i32(slots)
        _lib.check(self.lib.shahd_reset(self.handle, s.ctypes.data_as(_ip), s.size))

    def length(self, slot: int) -> int:
        n = self.lib.shahd_seq_length(self.handle, slot)
        if n < 0:
            _lib.check(n)
        return int(n)

    def prefill(self, slots, prompts) -> None:
        """PrefillCache for each slot (reset, then positions 0..len-1)."""
        s = _i32(slots)
        flat, offs = _pack(prompts)
        _lib.check(self.lib.shahd_prefill(self.handle, s.ctypes.data_as(_ip), flat.ctypes.data_as(_ip),
                                          offs.ctypes.data_as(_ip), s.size))

    def step(self, slots, tokens, want_logits: bool = True) -> tuple[np.ndarray | None, np.ndarray]:
        """CachedForwardStep for each (slot, token): returns (logits [n, V] or None, greedy ids [n])."""
        s, t = _i32(slots), _i32(tokens)
        n = s.size
        logits = np.empty((n, self.cfg.vocab_size), dtype=np.float32) if want_logits else None
        nxt = np.empty(n, dtype=np.int32)
        _lib.check(self.lib.shahd_step(self.handle, s.ctypes.data_as(_ip), t.ctypes.data_as(_ip), n,
                                       logits.ctypes.data_as(_fp) if logits is not None else None,
                                       nxt.ctypes.data_as(_ip)))
        return logits, nxt

    def verify(self, slots, token_lists, want_logits: bool = False):
        """Append each slot's tokens at its cached length with the LM head on every row (the target pass
        of speculative decoding). Returns per slot the greedy id after each appended token (and the
        logits rows when asked)."""
        flat, offs = _pack(token_lists)
        sl = _i32(slots)
        ids = np.zeros(flat.size, dtype=np.int32)
        logits = np.zeros((flat.size, self.cfg.vocab_size), dtype=np.float32) if want_logits else None
        _lib.check(self.lib.shahd_verify(self.handle, sl.ctypes.data_as(_ip), flat.ctypes.data_as(_ip),
                                         offs.ctypes.data_as(_ip), sl.size,
                                         logits.ctypes.data_as(_fp) if logits is not None else None,
                                         ids.ctypes.data_as(_ip)))
        out_ids = [ids[offs[i]:offs[i + 1]] for i in range(sl.size)]
        if want_logits:
            return out_ids, [logits[offs[i]:offs[i + 1]] for i in range(sl.size)]
        return out_ids

    def truncate(self, slots, lengths) -> None:
        """Keep only the first lengths[i] cached positions of each slot."""
        sl, ln = _i32(slots), _i32(lengths)
        _lib.check(self.lib.shahd_truncate(self.handle, sl.ctypes.data_as(_ip), ln.ctypes.data_as(_ip), sl.size))

    def generate(self, prompts, max_new: int, sampling: Sampling = GREEDY, rng_states=None) -> np.ndarray:
        """CachedGenerate for each prompt (slots 0..n-1): returns the new ids [n, max_new].

        With sampling.temperature > 0, rng_states (uint32 [n], one SeededRng state per sequence) is
        required; a uint32 array is advanced in place, as the reference's Rng object is."""
        flat, offs = _pack(prompts)
        n = offs.size - 1
        out = np.zeros((n, max(max_new, 0)), dtype=np.int32)
        st = np.ones(n, dtype=np.uint32) if rng_states is None else np.ascontiguousarray(rng_states, dtype=np.uint32)
        o = sampling.to_c()
        _lib.check(self.lib.shahd_generate(self.handle, flat.ctypes.data_as(_ip), offs.ctypes.data_as(_ip), n, max_new,
                                           ctypes.byref(o), st.ctypes.data_as(_up), out.ctypes.data_as(_ip)))
        if isinstance(rng_states, np.ndarray) and st is not rng_states:
            rng_states[...] = st  # SeededRng.SetState: the streams advanced by one draw per sampled token
        return out

    def generate_logits(self, prompts, max_new: int) -> tuple[np.ndarray, np.ndarray]:
        """Greedy CachedGenerate that also returns every step's logits [n, max_new, vocab] (the logits each
        new id was chosen from; CachedDecoder.Logits after each push). Needs the persistent decode loop."""
        flat, offs = _pack(prompts)
        n = offs.size - 1
        out = np.zeros((n, max(max_new, 0)), dtype=np.int32)
        logits = np.zeros((n, max(max_new, 0), self.cfg.vocab_size), dtype=np.float32)
        _lib.check(self.lib.shahd_generate_logits(self.handle, flat.ctypes.data_as(_ip), offs.ctypes.data_as(_ip), n,
                                                  max_new, out.ctypes.data_as(_ip), logits.ctypes.data_as(_fp)))
        return out, logits

    def generate_device(self, d_prompts: int, host_offsets: np.ndarray, max_new: int, d_out: int,
                        sampling: Sampling = GREEDY, d_rng: int = 0, stream: int = 0) -> None:
        """Asynchronous CachedGenerate over device buffers (ids already resident in HBM)."""
        offs = _i32(host_offsets)
        o = sampling.to_c()
        _lib.check(self.lib.shahd_generate_device(self.handle, ctypes.c_void_p(d_prompts), offs.ctypes.data_as(_ip),
                                                  offs.size - 1, max_new, ctypes.byref(o), ctypes.c_void_p(d_rng),
                                                  ctypes.c_void_p(d_out), ctypes.c_void_p(stream)))

    def sync(self) -> None:
        _lib.check(self.lib.shahd_sync(self.handle))

    def step_launches(self, n: int) -> int:
        return int(self.lib.shahd_step_launches(self.handle, n))

    def kernel_launches(self) -> int:
        return int(self.lib.shahd_kernel_launches(self.handle))

    def profile(self, enable: bool) -> None:
        _lib.check(self.lib.shahd_profile(self.handle, int(enable)))

    PROFILE_KINDS = {"attention": 0, "linear": 1, "other": 2,
                     "prefill_attention": 3, "prefill_linear": 4, "prefill_other": 5, "decode_loop": 6}

    def profile_read(self, kind: str) -> dict:
        ms = ctypes.c_double()
        n = ctypes.c_int64()
        b = ctypes.c_double()
        _lib.check(self.lib.shahd_profile_read(self.handle, self.PROFILE_KINDS[kind], ctypes.byref(ms), ctypes.byref(n),
                                               ctypes.byref(b)))
        return {"ms": ms.value, "launches": n.value, "bytes": b.value}


class CachedDecoder:
    """CachedDecoder (CachedForward.ts:113-150) over one slot: prefill the trailing window, keep the
    next-token logits, rebuild the cache from the last BlockSize-1 ids when it is full."""

    def __init__(self, session: Session, prompt_ids, slot: int = 0):
        prompt = [int(t) for t in prompt_ids]
        if not prompt:
            raise ValueError("CachedDecoder: empty prompt — nothing to condition on")
        self.s, self.slot = session, slot
        C = session.cfg.block_size
        context = prompt[-C:]
        session.prefill([slot], [context[:-1]])
        self.window = context[:-1]
        self.logits = self._step(context[-1])

    def _step(self, token: int) -> np.ndarray:
        logits, _ = self.s.step([self.slot], [token])
        self.window.append(token)
        return logits[0]

    def push(self, token: int) -> None:
        V = self.s.cfg.vocab_size
        if not (0 <= int(token) < V):
            raise ValueError(f"CachedDecoder.Push: token id {token} out of range [0,{V})")
        C = self.s.cfg.block_size
        if self.s.length(self.slot) >= C:
            keep = self.window[-(C - 1):]
            self.s.prefill([self.slot], [keep])
            self.window = list(keep)
        self.logits = self._step(int(token))


def sample_from_logits(logits, sampling: Sampling = GREEDY, rng_states=None) -> np.ndarray:
    """SampleFromLogits (Sampler.ts:16-27) for each row of logits [rows, vocab] on the GPU.

    With sampling.temperature > 0, rng_states (uint32 [rows]) is required and advanced in place by one
    draw per row. Returns the chosen ids [rows]."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    if lg.ndim == 1:
        lg = lg[None, :]
    rows, vocab = lg.shape
    out = np.zeros(rows, dtype=np.int32)
    st = None if rng_states is None else np.ascontiguousarray(rng_states, dtype=np.uint32)
    o = sampling.to_c()
    lib = _lib.load()
    _lib.check(lib.shahd_sample_logits(lg.ctypes.data_as(_fp), rows, vocab, ctypes.byref(o),
                                       st.ctypes.data_as(_up) if st is not None else None, out.ctypes.data_as(_ip)))
    if isinstance(rng_states, np.ndarray) and st is not rng_states:
        rng_states[...] = st
    return out


def cached_generate(session: Session, prompt_ids, max_new: int, sampling: Sampling = GREEDY, rng_state: int = 1):
    """CachedGenerate (CachedForward.ts:153-171) for one prompt; returns prompt + new ids."""
    prompt = [int(t) for t in prompt_ids]
    if not prompt:
        raise ValueError("CachedGenerate: empty prompt — nothing to condition on")
    if max_new < 1:
        return list(prompt)
    out = session.generate([prompt], max_new, sampling, np.array([rng_state], dtype=np.uint32))
    return prompt + out[0].tolist()
