"""Seed-generated TinyLlama weight archives and their INT8 quantization.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The real TinyLlama checkpoint is not available offline, so parity runs on a
random model drawn from a fixed seed. :func:`random_archive` produces a dict in
the reference's ``TinyLlamaWeights`` npz key schema (model/tinyllama.py:205-221
for the ``meta_*`` keys, :249-267 for the per-layer keys, :322-377 for how the
reference writes them): ``W`` is stored ``[in, out]`` so that ``x @ W`` is the
projection. Such a dict can be ``np.savez``'d and opened by the reference's own
``TinyLlamaWeights`` unchanged.

:func:`quantize_archive` turns it into INT8 weights plus one float64 scale per
output channel:
* ``granularity="tensor"`` reproduces the reference bridge, which quantizes
  each float weight per tensor on every call (model/tinyllama_gemm_int8.py:69);
  the per-tensor scale is broadcast over the output channels.
* ``granularity="channel"`` is the static per-output-channel scheme of the
  hardware spec (docs/design_decisions.txt, A10) and of benchmark config 0.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .golden import quantize_int8

TINYLLAMA = {
    "hidden_size": 2048,
    "intermediate_size": 5632,
    "num_hidden_layers": 22,
    "num_attention_heads": 32,
    "num_key_value_heads": 4,
    "head_dim": 64,
    "vocab_size": 32000,
    "max_position_embeddings": 2048,
    "rms_norm_eps": 1e-5,
    "rope_theta": 10000.0,
}

PROJ_NAMES = ("q", "k", "v", "o", "gate", "up", "down")


def full_cfg(base: dict) -> dict:
    """Add the derived keys the reference computes on load
    (model/tinyllama.py:218-221)."""
    cfg = dict(base)
    cfg["num_key_value_groups"] = cfg["num_attention_heads"] // cfg["num_key_value_heads"]
    cfg["attn_scale"] = 1.0 / np.sqrt(cfg["head_dim"])  # NumPy float64 scalar
    # The archive stores eps/theta as float32 (model/tinyllama.py:334-335).
    cfg["rms_norm_eps"] = float(np.float32(cfg["rms_norm_eps"]))
    cfg["rope_theta"] = float(np.float32(cfg["rope_theta"]))
    return cfg


def proj_shapes(cfg: dict) -> dict:
    d, f = cfg["hidden_size"], cfg["intermediate_size"]
    kv = cfg["num_key_value_heads"] * cfg["head_dim"]
    q = cfg["num_attention_heads"] * cfg["head_dim"]
    return {"q": (d, q), "k": (d, kv), "v": (d, kv), "o": (q, d),
            "gate": (d, f), "up": (d, f), "down": (f, d)}


def random_archive(seed: int, n_layers: int, dims: dict | None = None, std: float = 0.02,
                   gamma_one: bool = True) -> dict:
    """Random float32 archive: every matrix and the embedding table ~ N(0, std),
    RMSNorm gains 1 (or 1 + N(0, 0.1) with ``gamma_one=False``)."""
    base = dict(TINYLLAMA if dims is None else dims)
    base["num_hidden_layers"] = n_layers
    rng = np.random.default_rng(seed)
    d, v = base["hidden_size"], base["vocab_size"]
    shapes = proj_shapes(base)

    def normal(shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def gain():
        if gamma_one:
            return np.ones(d, dtype=np.float32)
        return (1.0 + 0.1 * rng.standard_normal(d, dtype=np.float32)).astype(np.float32)

    arc = {
        "meta_model_id": np.array("random-tinyllama"),
        "meta_hidden_size": np.array(base["hidden_size"], dtype=np.int32),
        "meta_intermediate_size": np.array(base["intermediate_size"], dtype=np.int32),
        "meta_num_hidden_layers": np.array(n_layers, dtype=np.int32),
        "meta_num_attention_heads": np.array(base["num_attention_heads"], dtype=np.int32),
        "meta_num_key_value_heads": np.array(base["num_key_value_heads"], dtype=np.int32),
        "meta_head_dim": np.array(base["head_dim"], dtype=np.int32),
        "meta_vocab_size": np.array(v, dtype=np.int32),
        "meta_max_position_embeddings": np.array(base["max_position_embeddings"], dtype=np.int32),
        "meta_rms_norm_eps": np.array(base["rms_norm_eps"], dtype=np.float32),
        "meta_rope_theta": np.array(base["rope_theta"], dtype=np.float32),
    }
    arc["embed_w"] = normal((v, d))
    for i in range(n_layers):
        for name in PROJ_NAMES:
            arc[f"layer{i}_{name}_w"] = normal(shapes[name])
        arc[f"layer{i}_input_norm_w"] = gain()
        arc[f"layer{i}_post_norm_w"] = gain()
    arc["final_norm_w"] = gain()
    arc["lm_head_w"] = normal((d, v))
    return arc


def archive_cfg(arc: dict) -> dict:
    """Config dict read back from the ``meta_*`` keys (model/tinyllama.py:205-217)."""
    base = {
        "hidden_size": int(arc["meta_hidden_size"]),
        "intermediate_size": int(arc["meta_intermediate_size"]),
        "num_hidden_layers": int(arc["meta_num_hidden_layers"]),
        "num_attention_heads": int(arc["meta_num_attention_heads"]),
        "num_key_value_heads": int(arc["meta_num_key_value_heads"]),
        "head_dim": int(arc["meta_head_dim"]),
        "vocab_size": int(arc["meta_vocab_size"]),
        "max_position_embeddings": int(arc["meta_max_position_embeddings"]),
        "rms_norm_eps": float(arc["meta_rms_norm_eps"]),
        "rope_theta": float(arc["meta_rope_theta"]),
    }
    return full_cfg(base)


@dataclass
class QLinear:
    w_q: np.ndarray        # int8 [in, out]
    scale: np.ndarray      # float64 [out]


@dataclass
class QLayer:
    q: QLinear
    k: QLinear
    v: QLinear
    o: QLinear
    gate: QLinear
    up: QLinear
    down: QLinear
    input_norm: np.ndarray
    post_norm: np.ndarray


@dataclass
class QModel:
    cfg: dict
    embed: np.ndarray                 # float32 [V, D]
    final_norm: np.ndarray            # float32 [D]
    lm_head: QLinear
    layers: list = field(default_factory=list)


def quantize_weight(w: np.ndarray, granularity: str) -> QLinear:
    """INT8 weight + float64 per-output-channel scale.

    ``tensor``: one :func:`quantize_int8` over the whole matrix, scale
    broadcast (bit-identical ``w_q`` to the reference bridge's call at
    model/tinyllama_gemm_int8.py:69). ``channel``: the same rule applied to
    each output column independently."""
    w = np.asarray(w, dtype=np.float32)
    n_out = w.shape[1]
    if granularity == "tensor":
        q, s = quantize_int8(w)
        return QLinear(q, np.full(n_out, s, dtype=np.float64))
    if granularity != "channel":
        raise ValueError(f"unknown granularity {granularity!r}")
    peak = np.max(np.abs(w), axis=0).astype(np.float64)
    scale = np.where(peak == 0.0, 1.0, peak / 127.0)
    q = np.empty(w.shape, dtype=np.int8)
    # Column-wise f32 division by f32(scale) with half-to-even rounding, as
    # quantize_int8 does for the whole tensor.
    q[:] = np.clip(np.round(w / scale.astype(np.float32)[np.newaxis, :]), -127, 127)
    return QLinear(q, scale)


def quantize_archive(arc: dict, granularity: str = "tensor") -> QModel:
    cfg = archive_cfg(arc)
    layers = []
    for i in range(cfg["num_hidden_layers"]):
        qs = {n: quantize_weight(arc[f"layer{i}_{n}_w"], granularity) for n in PROJ_NAMES}
        layers.append(QLayer(**qs,
                             input_norm=np.asarray(arc[f"layer{i}_input_norm_w"], np.float32),
                             post_norm=np.asarray(arc[f"layer{i}_post_norm_w"], np.float32)))
    return QModel(cfg=cfg,
                  embed=np.asarray(arc["embed_w"], np.float32),
                  final_norm=np.asarray(arc["final_norm_w"], np.float32),
                  lm_head=quantize_weight(arc["lm_head_w"], granularity),
                  layers=layers)


def small_dims(vocab: int = 512, hidden: int = 256, ffn: int = 704, heads: int = 4,
               kv_heads: int = 2, head_dim: int = 64, max_pos: int = 2048) -> dict:
    """A scaled-down TinyLlama shape for fast CPU fixtures (same head_dim,
    GQA ratio heads/kv_heads, SwiGLU, RMSNorm, RoPE)."""
    return {"hidden_size": hidden, "intermediate_size": ffn, "num_hidden_layers": 1,
            "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": head_dim,
            "vocab_size": vocab, "max_position_embeddings": max_pos,
            "rms_norm_eps": 1e-5, "rope_theta": 10000.0}


def random_qmodel(seed: int, n_layers: int, dims: dict | None = None, std: float = 0.02,
                  granularity: str = "channel") -> QModel:
    """A seeded random model drawn and quantized one matrix at a time, so a
    full 22-layer TinyLlama (1.04e9 INT8 weights) never holds its float
    weights at once: every matrix and the embedding table ~ N(0, std) in
    float32, quantized per output channel (or per tensor), RMSNorm gains 1.
    Same distribution as :func:`random_archive` followed by
    :func:`quantize_archive` (a different random stream)."""
    base = dict(TINYLLAMA if dims is None else dims)
    base["num_hidden_layers"] = n_layers
    cfg = full_cfg(base)
    rng = np.random.default_rng(seed)
    d, v = cfg["hidden_size"], cfg["vocab_size"]
    shapes = proj_shapes(cfg)

    def draw(shape):
        return quantize_weight(rng.standard_normal(shape, dtype=np.float32) * np.float32(std), granularity)

    layers = []
    for _ in range(n_layers):
        qs = {n: draw(shapes[n]) for n in PROJ_NAMES}
        layers.append(QLayer(**qs, input_norm=np.ones(d, np.float32), post_norm=np.ones(d, np.float32)))
    embed = (rng.standard_normal((v, d), dtype=np.float32) * np.float32(std)).astype(np.float32)
    return QModel(cfg=cfg, embed=embed, final_norm=np.ones(d, np.float32), lm_head=draw((d, v)), layers=layers)


class ArchiveWeights:
    """In-memory stand-in for the reference's ``TinyLlamaWeights`` over an
    archive dict from :func:`random_archive`: the same ``cfg`` keys and the
    same accessors (``embed``, ``final_norm_w``, ``lm_head_w``, ``layer`` with
    ``*_b`` entries None when absent, ``_array``), model/tinyllama.py:198-267,
    without writing the archive to disk."""

    def __init__(self, arc: dict):
        self.data = arc
        self.cfg = archive_cfg(arc)
        self.cfg["model_id"] = str(np.asarray(arc.get("meta_model_id", "random")).item())

    def _array(self, key: str) -> np.ndarray:
        return np.asarray(self.data[key], dtype=np.float32)

    def _optional_array(self, key: str):
        return self._array(key) if key in self.data else None

    def embed(self, token_ids) -> np.ndarray:
        return self._array("embed_w")[token_ids]

    def final_norm_w(self) -> np.ndarray:
        return self._array("final_norm_w")

    def lm_head_w(self) -> np.ndarray:
        return self._array("lm_head_w")

    def layer(self, idx: int) -> dict:
        d = {f"{p}_w": self._array(f"layer{idx}_{p}_w") for p in PROJ_NAMES}
        d.update({f"{p}_b": self._optional_array(f"layer{idx}_{p}_b") for p in PROJ_NAMES})
        d["input_norm_w"] = self._array(f"layer{idx}_input_norm_w")
        d["post_norm_w"] = self._array(f"layer{idx}_post_norm_w")
        return d
