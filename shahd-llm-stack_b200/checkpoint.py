"""Checkpoint -> device weights: serve a released Shahd checkpoint from a GPU session.

Mirrors Brain/Checkpoint/CheckpointFormat.ts (f64 tensors base64-encoded, sha256 payload checksum),
CheckpointReader.ts (ParseCheckpoint: version and checksum checks; ApplyParams: shape checks, then the
weights in Shahd.Parameters() order, Brain/Nn/Shahd.ts:87-94) and the Model section of the config the
checkpoint carries (Brain/Config/Constants.ts:11-26, DeriveConfig.ts:8-20). Only the weights are used:
a decode session needs no optimizer moments or training RNG state (ApplyCheckpointWeights,
CheckpointReader.ts:71-73).

The checksum hashes JSON.stringify(Config), so the config is re-serialized with JavaScript's number and
string formatting (js_stringify) to reproduce the writer's bytes.
"""
from __future__ import annotations

import base64
import hashlib
import json
import math

import numpy as np

from .decode import ModelConfig, Session

FORMAT_VERSION = 1  # CheckpointFormat.ts:9
SHAPE_FIELDS = ("EmbedDim", "NumLayers", "NumHeads", "BlockSize", "VocabSize")  # CheckpointReader.ts:12


class CheckpointError(ValueError):
    pass


# ---- JSON.stringify ----------------------------------------------------------------------------------

def js_number(x) -> str:
    """Number::toString of ECMAScript as JSON.stringify prints it (shortest round-trip digits; plain
    notation for decimal exponents -6 .. 20, exponent form otherwise; NaN and infinities -> null)."""
    if isinstance(x, bool):
        raise TypeError("bool is not a number")
    if isinstance(x, int):
        return str(x)
    if math.isnan(x) or math.isinf(x):
        return "null"
    if x == 0:
        return "0"
    sign = "-" if x < 0 else ""
    r = repr(abs(float(x)))
    mant, exp = (r.split("e") + ["0"])[:2]
    exp = int(exp)
    ip, fp = (mant.split(".") + [""])[:2]
    if ip.strip("0"):
        n = len(ip.lstrip("0")) + exp  # value = 0.DIGITS x 10^n
    else:
        n = exp - (len(fp) - len(fp.lstrip("0")))
    digits = (ip + fp).lstrip("0").rstrip("0") or "0"
    k = len(digits)
    if k <= n <= 21:
        s = digits + "0" * (n - k)
    elif 0 < n <= 21:
        s = digits[:n] + "." + digits[n:]
    elif -6 < n <= 0:
        s = "0." + "0" * (-n) + digits
    else:
        e = n - 1
        s = digits[0] + ("." + digits[1:] if k > 1 else "") + "e" + ("+" if e >= 0 else "-") + str(abs(e))
    return sign + s


def js_stringify(v) -> str:
    """JSON.stringify(v) with no indentation, keys in insertion order."""
    if v is None:
        return "null"
    if v is True:
        return "true"
    if v is False:
        return "false"
    if isinstance(v, (int, float)):
        return js_number(v)
    if isinstance(v, str):
        return json.dumps(v, ensure_ascii=False)
    if isinstance(v, (list, tuple)):
        return "[" + ",".join(js_stringify(x) for x in v) + "]"
    if isinstance(v, dict):
        return "{" + ",".join(json.dumps(str(k), ensure_ascii=False) + ":" + js_stringify(x) for k, x in v.items()) + "}"
    raise TypeError(f"cannot serialize {type(v).__name__}")


# ---- payload ----------------------------------------------------------------------------------------

def encode_float64(a) -> str:
    """EncodeFloat64 (CheckpointFormat.ts:49-52): the raw little-endian f64 bytes, f32 widened first."""
    return base64.b64encode(np.ascontiguousarray(a, dtype="<f8").tobytes()).decode("ascii")


def decode_float64(b64: str) -> np.ndarray:
    """DecodeFloat64 (CheckpointFormat.ts:55-60)."""
    return np.frombuffer(base64.b64decode(b64), dtype="<f8").copy()


def checksum_payload(params: list, optimizer: dict, config: dict) -> str:
    """ChecksumPayload (CheckpointFormat.ts:32-43): sha256 over each tensor's "RxC:" + data, the
    optimizer moments, the step count and JSON.stringify(Config)."""
    h = hashlib.sha256()
    for p in params:
        h.update(f"{p['Rows']}x{p['Cols']}:".encode())
        h.update(p["Data"].encode())
    for m in optimizer.get("M", []):
        h.update(m.encode())
    for v in optimizer.get("V", []):
        h.update(v.encode())
    h.update(js_number(optimizer.get("StepCount", 0)).encode())
    h.update(js_stringify(config).encode())
    return h.hexdigest()


# ---- reading ----------------------------------------------------------------------------------------

def parse_checkpoint(text: str) -> dict:
    """ParseCheckpoint (CheckpointReader.ts:17-29): format version, then the checksum when present."""
    data = json.loads(text)
    if data.get("FormatVersion") != FORMAT_VERSION:
        raise CheckpointError(f"ParseCheckpoint: format version {data.get('FormatVersion')} != {FORMAT_VERSION}")
    if isinstance(data.get("Checksum"), str):
        actual = checksum_payload(data["Params"], data["Optimizer"], data["Config"])
        if actual != data["Checksum"]:
            raise CheckpointError("ParseCheckpoint: checksum mismatch — checkpoint is corrupt or truncated "
                                  f"(expected {data['Checksum'][:12]}…, got {actual[:12]}…)")
    return data


def load_checkpoint(path: str) -> dict:
    with open(path, encoding="utf-8") as f:
        return parse_checkpoint(f.read())


def model_config_from(config: dict) -> ModelConfig:
    """The decode-relevant Model knobs of a checkpoint's config (Constants.ts:11-26), with Derived
    values resolved like DeriveConfig.ts:8-20 (MlpHidden = Math.round(EmbedDim * MlpRatio))."""
    m = config["Model"]
    e = int(m["EmbedDim"])
    return ModelConfig(
        embed_dim=e, num_layers=int(m["NumLayers"]), num_heads=int(m["NumHeads"]), block_size=int(m["BlockSize"]),
        vocab_size=int(m["VocabSize"]), mlp_hidden=int(math.floor(e * float(m.get("MlpRatio", 4)) + 0.5)),
        kv_heads=m.get("KvHeads"), position_scheme=m.get("PositionScheme", "Learned"),
        norm_kind=m.get("NormKind", "LayerNorm"), mlp_kind=m.get("MlpKind", "Relu"),
        weight_tying=bool(m.get("WeightTying", True)), layer_norm_eps=float(m.get("LayerNormEps", 1e-5)))


def param_shapes(cfg: ModelConfig) -> list[tuple[int, int]]:
    """[Rows, Cols] of every tensor of Shahd.Parameters() (Shahd.ts:87-94; Embedding.ts:28-30,
    Block.ts:34-41, NormLayer.ts:28-30, MultiHeadAttention.ts:76-78, Mlp.ts:59-65)."""
    E, V, C, F, d = cfg.embed_dim, cfg.vocab_size, cfg.block_size, cfg.mlp_hidden, cfg.head_dim
    norm = [(1, E), (1, E)] if cfg.norm_kind == "LayerNorm" else [(1, E)]
    out = [(V, E)] + ([(C, E)] if cfg.position_scheme == "Learned" else [])
    for _ in range(cfg.num_layers):
        out += norm
        out += [(E, d)] * cfg.num_heads + [(E, d)] * cfg.kv + [(E, d)] * cfg.kv + [(d, E)] * cfg.num_heads
        out += norm
        if cfg.mlp_kind == "Relu":
            out += [(E, F), (1, F), (F, E), (1, E)]
        else:
            out += [(E, F), (E, F), (F, E)]
    out += norm
    if not cfg.weight_tying:
        out.append((E, V))
    out.append((1, V))
    return out


def checkpoint_params(ckpt: dict, cfg: ModelConfig) -> np.ndarray:
    """ApplyParams (CheckpointReader.ts:37-64): the architecture fields must match, then every tensor's
    shape and payload length; returns the weights flattened in Parameters() order (f64)."""
    m = ckpt["Config"]["Model"]
    have = {"EmbedDim": cfg.embed_dim, "NumLayers": cfg.num_layers, "NumHeads": cfg.num_heads,
            "BlockSize": cfg.block_size, "VocabSize": cfg.vocab_size}
    diffs = [f"{k}: checkpoint={m.get(k)} model={have[k]}" for k in SHAPE_FIELDS if m.get(k) != have[k]]
    if diffs:
        raise CheckpointError("ApplyCheckpoint: architecture mismatch — cannot load weights:\n  " + "\n  ".join(diffs))
    shapes = param_shapes(cfg)
    if len(shapes) != len(ckpt["Params"]):
        raise CheckpointError(f"ApplyCheckpoint: parameter count mismatch {len(shapes)} vs {len(ckpt['Params'])}")
    parts = []
    for i, ((r, c), p) in enumerate(zip(shapes, ckpt["Params"])):
        if p["Rows"] != r or p["Cols"] != c:
            raise CheckpointError(f"ApplyCheckpoint: tensor {i} shape {r}x{c} vs {p['Rows']}x{p['Cols']}")
        a = decode_float64(p["Data"])
        if a.size != r * c:
            raise CheckpointError(f"ApplyCheckpoint: tensor {i} payload length {a.size} != {r * c} "
                                  "(truncated/corrupt checkpoint)")
        parts.append(a)
    return np.concatenate(parts)


def session_from_checkpoint(ckpt, max_seqs: int, device: int = 0, kv_pages: int = 0) -> tuple[Session, ModelConfig]:
    """A GPU session holding a checkpoint's weights (a path, the checkpoint text, or a parsed dict)."""
    if isinstance(ckpt, str):
        ckpt = parse_checkpoint(ckpt) if ckpt.lstrip().startswith("{") else load_checkpoint(ckpt)
    cfg = model_config_from(ckpt["Config"])
    return Session(cfg, checkpoint_params(ckpt, cfg), max_seqs, device=device, kv_pages=kv_pages), cfg


# ---- writing (weights only) ---------------------------------------------------------------------------

def build_checkpoint(config: dict, params: np.ndarray, cfg: ModelConfig, config_hash: str = "",
                     meta: dict | None = None) -> dict:
    """BuildCheckpoint (CheckpointWriter.ts:29-65) for weights only: empty optimizer state, zero RNG
    states, with the payload checksum. `config` is the full config object the checkpoint embeds."""
    flat = np.ascontiguousarray(params, dtype=np.float64)
    tensors, off = [], 0
    for r, c in param_shapes(cfg):
        tensors.append({"Rows": r, "Cols": c, "Data": encode_float64(flat[off:off + r * c])})
        off += r * c
    if off != flat.size:
        raise CheckpointError(f"build_checkpoint: {flat.size} parameters for a model of {off}")
    optimizer = {"M": [], "V": [], "StepCount": 0}
    ck = {"FormatVersion": FORMAT_VERSION, "ConfigHash": config_hash, "Config": config, "Params": tensors,
          "Optimizer": optimizer, "Rng": {"Init": 0, "Data": 0, "Dropout": 0, "Sampling": 0},
          "TokenizerState": None, "Meta": meta or {}}
    ck["Checksum"] = checksum_payload(tensors, optimizer, config)
    return ck
