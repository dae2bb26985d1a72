"""ctypes binding of ``libtl_b200.so`` (include/tl_api.h) and a Python surface
that mirrors the reference's own operator API.

Reference entry points mirrored here (same names, same argument meaning, same
error behaviour where the reference has one):

* ``quantized_linear(x, w, b=None, capture_arrays=False)``
  model/tinyllama_gemm_int8.py:59-88 -> returns ``(out, debug)`` with the
  same debug keys (``input_q``, ``weight_q``, ``accum_int32``,
  ``input_scale``, ``weight_scale``).
* ``quantize_int8(t)``           model/tinyllama_gemm_int8.py:36-42
* ``rms_norm(x, w, eps)``        model/tinyllama.py:45-50
* ``forward_mixed(token_ids, weights, cos, sin, layer_count, quantize_lm_head)``
  model/tinyllama_gemm_int8.py:437-467 -> logits of every row, [S, vocab]
* ``mixed_precision_decoder_layer(x, layer, cfg, cos, sin, capture_arrays)``
  model/tinyllama_gemm_int8.py:256-281 -> ``(out, debug)`` with the
  reference's nested debug keys (``Engine.decoder_layer`` for a loaded model)
* ``Engine.generate`` / ``generate_batch``: run_generate
  (model/tinyllama_gemm_int8.py:629-685) with the RTL launch/stop contract
  (rtl/control/prefill_decode_controller.sv, stop_condition_unit.sv).

Every computation runs in the CUDA library; there is no CPU path. If the
library is missing or no GPU is visible, calls raise.
"""

from __future__ import annotations

import ctypes as C
from collections import OrderedDict
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libtl_b200.so"

TL_OK = 0
STATUS_NAMES = {
    0: "TL_OK", 1: "TL_ERR_BAD_DESCRIPTOR", 2: "TL_ERR_HBM_READ", 3: "TL_ERR_HBM_WRITE",
    4: "TL_ERR_SCALE_METADATA", 5: "TL_ERR_DEBUG_OVERFLOW", 6: "TL_ERR_UNSUPPORTED_MODE",
    7: "TL_ERR_INTERNAL", 16: "TL_ERR_INVALID_ARGUMENT", 17: "TL_ERR_OUT_OF_RANGE",
    18: "TL_ERR_CUDA", 19: "TL_ERR_NCCL", 20: "TL_ERR_TIMEOUT", 21: "TL_ERR_NOT_LOADED",
    22: "TL_ERR_UNIMPLEMENTED",
}
STOP_NONE, STOP_EOS, STOP_MAX_TOKENS, STOP_HOST_ABORT, STOP_INTERNAL_ERR = 0, 1, 2, 3, 4
MODE_PREFILL, MODE_DECODE = 0, 1

# Every symbol the header declares (checked by the CPU tests).
EXPORTS = (
    "tl_status_string", "tl_version", "tl_create", "tl_destroy", "tl_tp_unique_id", "tl_tp_create", "tl_tp_create_ex",
    "tl_load_weights",
    "tl_init_random_weights", "tl_generate", "tl_generate_batch", "tl_abort",
    "tl_prefill_logits", "tl_decode_logits", "tl_read_kv", "tl_get_position",
    "tl_decode_steps_device", "tl_prefill_batch_device", "tl_decode_rewind", "tl_synchronize",
    "tl_decode_step_kernel_count", "tl_decode_step_kernel_count_rows", "tl_decode_row_groups", "tl_engine_stream", "tl_profile_decode_kernels", "tl_device_error",
    "tl_transpose_i8", "tl_quantize_int8",
    "tl_gemm_i8", "tl_gemm_i8_requant", "tl_quantized_linear", "tl_rmsnorm", "tl_lmhead_argmax",
    "tl_attn_decode", "tl_attn_prefill", "tl_lmhead_argmax_noalloc",
    "tl_forward_logits", "tl_decoder_layer", "tl_decode_layer", "tl_decode_debug",
    "tl_contract_rmsnorm", "tl_contract_silu", "tl_contract_softmax", "tl_contract_rope", "tl_residual_add_i32",
)


class TLError(RuntimeError):
    def __init__(self, code: int, what: str, detail: str = ""):
        self.code = code
        super().__init__(f"{what}: {STATUS_NAMES.get(code, code)} {detail}".rstrip())


class Config(C.Structure):
    _fields_ = [("hidden_size", C.c_int32), ("intermediate_size", C.c_int32),
                ("num_layers", C.c_int32), ("num_heads", C.c_int32), ("num_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("vocab_size", C.c_int32), ("max_positions", C.c_int32),
                ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float), ("max_batch", C.c_int32),
                ("max_prefill_tokens", C.c_int32)]


class LinearView(C.Structure):
    _fields_ = [("w", C.c_void_p), ("scale", C.c_void_p)]


class LayerView(C.Structure):
    _fields_ = [("q", LinearView), ("k", LinearView), ("v", LinearView), ("o", LinearView),
                ("gate", LinearView), ("up", LinearView), ("down", LinearView),
                ("input_norm", C.c_void_p), ("post_norm", C.c_void_p)]


class WeightsView(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("final_norm", C.c_void_p), ("lm_head", LinearView),
                ("layers", C.POINTER(LayerView)), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p)]


class RunStatus(C.Structure):
    _fields_ = [("status_word", C.c_uint32), ("generated_count", C.c_uint32),
                ("last_token", C.c_uint32), ("current_layer", C.c_uint32),
                ("current_block", C.c_uint32), ("stop_reason", C.c_int32),
                ("error_code", C.c_int32), ("position", C.c_uint32)]

    def as_dict(self) -> dict:
        return {f: getattr(self, f) for f, _ in self._fields_}


# tl_layer_capture: (field, element dtype, shape key) in the C struct's order.
# Shape keys: S rows, D hidden, Dq heads*64, Dkv kv_heads*64, F intermediate,
# HSS heads x S x S, 1 one float.
CAPTURE_FIELDS = (
    ("attn_input", np.float32, "SD"), ("qkv_input_q", np.int8, "SD"), ("qkv_input_absmax", np.float32, "1"),
    ("q_acc", np.int32, "SDq"), ("k_acc", np.int32, "SDkv"), ("v_acc", np.int32, "SDkv"),
    ("q_proj", np.float32, "SDq"), ("k_proj", np.float32, "SDkv"), ("v_proj", np.float32, "SDkv"),
    ("scores", np.float32, "HSS"), ("probs", np.float32, "HSS"), ("attended", np.float32, "SDq"),
    ("o_input_q", np.int8, "SDq"), ("o_input_absmax", np.float32, "1"), ("o_acc", np.int32, "SD"),
    ("o_proj", np.float32, "SD"), ("x_after_attn", np.float32, "SD"), ("ffn_input", np.float32, "SD"),
    ("gate_up_input_q", np.int8, "SD"), ("gate_up_input_absmax", np.float32, "1"),
    ("gate_acc", np.int32, "SF"), ("up_acc", np.int32, "SF"), ("gate_proj", np.float32, "SF"),
    ("up_proj", np.float32, "SF"), ("hidden", np.float32, "SF"), ("down_input_q", np.int8, "SF"),
    ("down_input_absmax", np.float32, "1"), ("down_acc", np.int32, "SD"), ("down_proj", np.float32, "SD"),
)


class LayerCapture(C.Structure):
    _fields_ = [(name, C.c_void_p) for name, _, _ in CAPTURE_FIELDS]


# tl_debug_record pointer fields: (name, dtype, shape key); D hidden, Dq, Dkv,
# Hkv64 [kv_heads, 64], Hkv [kv_heads], Hn [heads, position + 1].
DEBUG_FIELDS = (
    ("layer_input", np.float32, "D"), ("qkv_input_q", np.int8, "D"), ("q_proj", np.float32, "Dq"),
    ("k_proj", np.float32, "Dkv"), ("v_proj", np.float32, "Dkv"), ("scores", np.float32, "Hn"),
    ("probs", np.float32, "Hn"), ("k_row", np.int8, "Hkv64"), ("v_row", np.int8, "Hkv64"),
    ("k_scale", np.float32, "Hkv"), ("v_scale", np.float32, "Hkv"), ("attended", np.float32, "Dq"),
    ("layer_output", np.float32, "D"), ("final_hidden", np.float32, "D"),
)


class DebugRecord(C.Structure):
    _fields_ = [("position", C.c_uint32), ("chosen_token", C.c_uint32), ("top_ids", C.c_uint32 * 16),
                ("top_logits", C.c_float * 16), ("input_absmax", C.c_float * 5)] + \
               [(name, C.c_void_p) for name, _, _ in DEBUG_FIELDS]


_LIB = None


def load_library(path: Path | str | None = None):
    """Load libtl_b200.so (built in-tree by build.py). Raises if it is missing."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"{p} not found: build it with build.py (nvcc, sm_100a); "
                          "there is no CPU fallback")
    lib = C.CDLL(str(p))
    vp, i32, u32, u64 = C.c_void_p, C.c_int32, C.c_uint32, C.c_uint64
    sig = {
        "tl_status_string": (C.c_char_p, [i32]),
        "tl_version": (i32, []),
        "tl_create": (i32, [C.POINTER(Config), i32, C.POINTER(vp)]),
        "tl_destroy": (i32, [vp]),
        "tl_tp_unique_id": (i32, [vp]),
        "tl_tp_create": (i32, [C.POINTER(Config), i32, i32, i32, vp, C.POINTER(vp)]),
        "tl_tp_create_ex": (i32, [C.POINTER(Config), i32, i32, i32, vp, i32, C.POINTER(vp)]),
        "tl_load_weights": (i32, [vp, C.POINTER(WeightsView)]),
        "tl_init_random_weights": (i32, [vp, u64]),
        "tl_generate": (i32, [vp, vp, u32, u32, u32, u32, vp, u32, C.POINTER(RunStatus)]),
        "tl_generate_batch": (i32, [vp, u32, vp, u32, u32, u32, vp, u32, vp]),
        "tl_abort": (i32, [vp]),
        "tl_prefill_logits": (i32, [vp, u32, vp, u32, vp]),
        "tl_decode_logits": (i32, [vp, u32, u32, vp]),
        "tl_read_kv": (i32, [vp, u32, u32, u32, vp, vp, vp, vp]),
        "tl_get_position": (i32, [vp, u32, C.POINTER(u32)]),
        "tl_decode_steps_device": (i32, [vp, u32, u32]),
        "tl_prefill_batch_device": (i32, [vp, u32, vp, u32]),
        "tl_decode_rewind": (i32, [vp, u32, u32]),
        "tl_synchronize": (i32, [vp]),
        "tl_decode_step_kernel_count": (i32, [vp]),
        "tl_decode_step_kernel_count_rows": (i32, [vp, u32]),
        "tl_decode_row_groups": (i32, [vp, u32]),
        "tl_engine_stream": (vp, [vp]),
        "tl_profile_decode_kernels": (i32, [vp, u32, u32, vp]),
        "tl_device_error": (i32, []),
        "tl_transpose_i8": (i32, [vp, vp, i32, i32, vp]),
        "tl_quantize_int8": (i32, [vp, i32, i32, i32, vp, vp, vp]),
        "tl_gemm_i8": (i32, [vp, vp, vp, i32, i32, i32, vp]),
        "tl_gemm_i8_requant": (i32, [vp, vp, vp, i32, i32, vp, i32, i32, i32, vp]),
        "tl_quantized_linear": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, vp]),
        "tl_rmsnorm": (i32, [vp, vp, C.c_float, vp, i32, i32, vp]),
        "tl_lmhead_argmax": (i32, [vp, vp, C.c_float, vp, vp, i32, i32, i32, vp, vp, vp]),
        "tl_attn_decode": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp]),
        "tl_attn_prefill": (i32, [vp, i32, i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp]),
        "tl_lmhead_argmax_noalloc": (i32, [vp, vp, C.c_float, vp, vp, i32, i32, i32, vp, vp, vp]),
        "tl_forward_logits": (i32, [vp, vp, u32, vp, vp]),
        "tl_decoder_layer": (i32, [vp, u32, u32, vp, u32, vp, C.POINTER(LayerCapture)]),
        "tl_decode_layer": (i32, [vp, u32, u32, vp, vp, vp, vp, C.POINTER(LayerCapture)]),
        "tl_decode_debug": (i32, [vp, u32, u32, u32, C.POINTER(DebugRecord), vp]),
        "tl_contract_rmsnorm": (i32, [vp, i32, i32, u32, vp, C.c_float, u32, vp, vp, vp]),
        "tl_contract_silu": (i32, [vp, C.c_int64, u32, u32, vp, vp, vp]),
        "tl_contract_softmax": (i32, [vp, i32, i32, u32, vp, vp, vp]),
        "tl_contract_rope": (i32, [vp, vp, vp, i32, vp, vp]),
        "tl_residual_add_i32": (i32, [vp, vp, vp, C.c_int64, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def check(code: int, what: str):
    if code != TL_OK:
        detail = ""
        try:
            detail = load_library().tl_status_string(code).decode()
        except Exception:
            pass
        raise TLError(code, what, detail)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# --------------------------------------------------------------------------
# Host-side model container (reference key schema, quantized)
# --------------------------------------------------------------------------
@dataclass
class Linear:
    w: np.ndarray       # int8 [in, out]
    scale: np.ndarray   # float64 [out]


@dataclass
class Layer:
    q: Linear
    k: Linear
    v: Linear
    o: Linear
    gate: Linear
    up: Linear
    down: Linear
    input_norm: np.ndarray
    post_norm: np.ndarray


@dataclass
class Model:
    cfg: dict
    embed: np.ndarray
    final_norm: np.ndarray
    lm_head: Linear
    layers: list = field(default_factory=list)


def quantize_weight(w: np.ndarray, granularity: str = "tensor") -> Linear:
    """INT8 weight with a float64 scale per output channel. ``tensor`` is the
    reference bridge's per-call rule (model/tinyllama_gemm_int8.py:36-42, 69),
    ``channel`` applies the same rule per output column."""
    w = np.asarray(w, dtype=np.float32)
    if granularity == "tensor":
        peak = float(np.max(np.abs(w))) if w.size else 0.0
        s = 1.0 if peak == 0.0 else peak / 127.0
        q = np.clip(np.round(w / s), -127, 127).astype(np.int8)
        return Linear(q, np.full(w.shape[1], s, dtype=np.float64))
    peak = np.max(np.abs(w), axis=0).astype(np.float64)
    s = np.where(peak == 0.0, 1.0, peak / 127.0)
    q = np.clip(np.round(w / s.astype(np.float32)[None, :]), -127, 127).astype(np.int8)
    return Linear(q, s)


def from_tinyllama_weights(weights, layer_count: int | None = None, granularity: str = "tensor") -> Model:
    """Quantize a reference ``TinyLlamaWeights``-like object (``cfg`` dict,
    ``layer(i)`` dict with ``q_w``.. ``down_w`` [in, out], norms, ``embed``,
    ``final_norm_w()``, ``lm_head_w()``; model/tinyllama.py:198-267)."""
    cfg = dict(weights.cfg)
    n = cfg["num_hidden_layers"] if layer_count is None else layer_count
    layers = []
    for i in range(n):
        d = weights.layer(i)
        layers.append(Layer(*(quantize_weight(d[f"{p}_w"], granularity)
                               for p in ("q", "k", "v", "o", "gate", "up", "down")),
                            input_norm=np.asarray(d["input_norm_w"], np.float32),
                            post_norm=np.asarray(d["post_norm_w"], np.float32)))
    emb = weights._array("embed_w") if hasattr(weights, "_array") else weights.embed_w
    cfg["num_hidden_layers"] = n
    return Model(cfg, np.asarray(emb, np.float32), np.asarray(weights.final_norm_w(), np.float32),
                 quantize_weight(weights.lm_head_w(), granularity), layers)


# meta_* keys of the reference's weight archive and the engine config keys
# they fill (model/tinyllama.py:322-335 writes them, :205-217 reads them)
_NPZ_META = (("hidden_size", int), ("intermediate_size", int), ("num_hidden_layers", int),
             ("num_attention_heads", int), ("num_key_value_heads", int), ("head_dim", int),
             ("vocab_size", int), ("max_position_embeddings", int), ("rms_norm_eps", float),
             ("rope_theta", float))
_NPZ_PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def checkpoint_config(arrays) -> dict:
    """Engine config from the ``meta_*`` entries of a weight archive in the
    reference's npz schema (``save_weights_from_hf``, model/tinyllama.py:292-382).
    ``arrays`` is the opened archive (or any mapping of the same keys)."""
    missing = [k for k, _ in _NPZ_META if f"meta_{k}" not in arrays]
    if missing:
        raise ValueError(f"not a TinyLlama weight archive: missing meta_{missing[0]}")
    cfg = {k: conv(np.asarray(arrays[f"meta_{k}"]).item()) for k, conv in _NPZ_META}
    if "meta_model_id" in arrays:
        cfg["model_id"] = str(np.asarray(arrays["meta_model_id"]).item())
    return cfg


def load_checkpoint_npz(path, layer_count: int | None = None, granularity: str = "channel") -> Model:
    """Read a weight archive written by the reference's ``save_weights_from_hf``
    (model/tinyllama.py:292-382: float16 or float32 arrays, projections stored
    ``[in, out]``, ``lm_head_w`` transposed to ``[hidden, vocab]``) and quantize
    it for :meth:`Engine.load`: every projection and the LM head to INT8 with a
    float64 scale per output channel (``granularity="channel"``, the hardware's
    static scheme) or per tensor (``"tensor"``, the reference bridge's per-call
    rule), norms and the embedding table as float32. The engine has no bias
    path (TinyLlama has none): an archive with ``layer*_b`` arrays is refused.
    ``layer_count`` keeps only the first layers."""
    with np.load(path, allow_pickle=False) as arrays:
        cfg = checkpoint_config(arrays)
        biases = sorted(k for k in arrays.files if k.startswith("layer") and k.endswith("_b"))
        if biases:
            raise ValueError(f"projection biases are not supported by the engine ({biases[0]})")
        n = cfg["num_hidden_layers"] if layer_count is None else int(layer_count)
        if not 0 < n <= cfg["num_hidden_layers"]:
            raise ValueError(f"layer_count {n} outside 1..{cfg['num_hidden_layers']}")
        shapes = model_shapes(cfg)
        d, v = cfg["hidden_size"], cfg["vocab_size"]
        expect = {"embed_w": (v, d), "final_norm_w": (d,), "lm_head_w": (d, v)}
        for i in range(n):
            expect.update({f"layer{i}_{p}_w": shapes[p] for p in _NPZ_PROJ})
            expect[f"layer{i}_input_norm_w"] = (d,)
            expect[f"layer{i}_post_norm_w"] = (d,)
        for key, shape in expect.items():
            if key not in arrays:
                raise ValueError(f"weight archive has no {key}")
            if tuple(arrays[key].shape) != shape:
                raise ValueError(f"{key}: shape {tuple(arrays[key].shape)}, the meta_* entries imply {shape}")
        layers = []
        for i in range(n):
            projs = [quantize_weight(arrays[f"layer{i}_{p}_w"], granularity) for p in _NPZ_PROJ]
            layers.append(Layer(*projs, input_norm=np.asarray(arrays[f"layer{i}_input_norm_w"], np.float32),
                                post_norm=np.asarray(arrays[f"layer{i}_post_norm_w"], np.float32)))
        cfg["num_hidden_layers"] = n
        return Model(cfg, np.asarray(arrays["embed_w"], np.float32), np.asarray(arrays["final_norm_w"], np.float32),
                     quantize_weight(arrays["lm_head_w"], granularity), layers)


def rope_tables(n_pos: int, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """float32 RoPE tables with the reference's NumPy arithmetic
    (model/tinyllama.py:59-66), so the device sees identical cos/sin."""
    inv_freq = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    ang = np.outer(np.arange(n_pos, dtype=np.float32), inv_freq)
    ang = np.concatenate([ang, ang], axis=-1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


_CFG_KEYS = ("hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
             "num_key_value_heads", "head_dim", "vocab_size", "max_position_embeddings")


def model_shapes(cfg: dict) -> dict:
    """[in, out] of each projection for a config (reference layout, x @ W)."""
    d, f = cfg["hidden_size"], cfg["intermediate_size"]
    dq = cfg["num_attention_heads"] * cfg["head_dim"]
    dkv = cfg["num_key_value_heads"] * cfg["head_dim"]
    return {"q": (d, dq), "k": (d, dkv), "v": (d, dkv), "o": (dq, d), "gate": (d, f), "up": (d, f), "down": (f, d)}


def check_model(model: Model, cfg: dict) -> None:
    """Raise ValueError unless every array of ``model`` has the shape the
    engine configuration ``cfg`` implies (and the model's own cfg agrees)."""
    for k in _CFG_KEYS:
        if int(model.cfg.get(k, -1)) != int(cfg[k]):
            raise ValueError(f"model {k}={model.cfg.get(k)} but the engine was created with {cfg[k]}")
    d, v = cfg["hidden_size"], cfg["vocab_size"]
    if len(model.layers) != cfg["num_hidden_layers"]:
        raise ValueError(f"model has {len(model.layers)} layers, engine expects {cfg['num_hidden_layers']}")

    def lin(name, l, shape):
        w = np.asarray(l.w)
        if w.shape != shape or w.dtype != np.int8:
            raise ValueError(f"{name}: weight {w.dtype} {w.shape}, expected int8 {shape}")
        if np.asarray(l.scale).shape != (shape[1],):
            raise ValueError(f"{name}: scale shape {np.asarray(l.scale).shape}, expected ({shape[1]},)")

    def vec(name, a, shape):
        if np.asarray(a).shape != shape:
            raise ValueError(f"{name}: shape {np.asarray(a).shape}, expected {shape}")

    shapes = model_shapes(cfg)
    for i, ly in enumerate(model.layers):
        for p in _NPZ_PROJ:
            lin(f"layer{i}.{p}", getattr(ly, p), shapes[p])
        vec(f"layer{i}.input_norm", ly.input_norm, (d,))
        vec(f"layer{i}.post_norm", ly.post_norm, (d,))
    vec("embed", model.embed, (v, d))
    vec("final_norm", model.final_norm, (d,))
    lin("lm_head", model.lm_head, (d, v))


# --------------------------------------------------------------------------
# Engine (runtime contract)
# --------------------------------------------------------------------------
TP_ID_BYTES = 128


def tp_unique_id() -> bytes:
    """NCCL group id for a tensor-parallel prefill group (drawn on rank 0 and
    handed to every rank's Engine(..., tp_id=...))."""
    lib = load_library()
    buf = (C.c_uint8 * TP_ID_BYTES)()
    check(lib.tl_tp_unique_id(C.addressof(buf)), "tl_tp_unique_id")
    return bytes(buf)


class Engine:
    """One engine per GPU: weights arena, INT8 KV cache for ``max_batch``
    sequences, captured decode graphs."""

    def __init__(self, cfg: dict, max_batch: int = 1, device: int = 0,
                 max_prefill_tokens: int | None = None, tp_rank: int = 0, tp_world: int = 1,
                 tp_id: bytes | None = None, tp_exchange: str = "allgather"):
        """``tp_world > 1`` makes rank ``tp_rank`` of a tensor-parallel
        prefill group (tl_tp_create_ex); every rank passes the same ``tp_id``
        from :func:`tp_unique_id` and all ranks construct concurrently.
        ``tp_exchange``: ``"allreduce"`` (O and down row-split, NCCL INT32
        all-reduce) or ``"allgather"`` (O and down replicated, INT8 inputs
        all-gathered by NVLink peer stores)."""
        self.lib = load_library()
        self.cfg = dict(cfg)
        c = Config(hidden_size=cfg["hidden_size"], intermediate_size=cfg["intermediate_size"],
                   num_layers=cfg["num_hidden_layers"], num_heads=cfg["num_attention_heads"],
                   num_kv_heads=cfg["num_key_value_heads"], head_dim=cfg["head_dim"],
                   vocab_size=cfg["vocab_size"], max_positions=cfg["max_position_embeddings"],
                   rms_norm_eps=cfg["rms_norm_eps"], rope_theta=cfg["rope_theta"],
                   max_batch=max_batch,
                   max_prefill_tokens=max_prefill_tokens or cfg["max_position_embeddings"])
        h = C.c_void_p()
        if tp_world > 1:
            if tp_id is None or len(tp_id) != TP_ID_BYTES:
                raise ValueError("tensor-parallel engines need the group's tp_unique_id() bytes")
            modes = {"allreduce": 0, "allgather": 1}
            if tp_exchange not in modes:
                raise ValueError(f"tp_exchange must be one of {sorted(modes)}")
            idbuf = (C.c_uint8 * TP_ID_BYTES).from_buffer_copy(tp_id)
            check(self.lib.tl_tp_create_ex(C.byref(c), device, tp_rank, tp_world, C.addressof(idbuf),
                                           modes[tp_exchange], C.byref(h)), "tl_tp_create_ex")
        else:
            check(self.lib.tl_create(C.byref(c), device, C.byref(h)), "tl_create")
        self.h = h
        self.tp_rank, self.tp_world = tp_rank, tp_world
        self.max_batch = max_batch
        self._keep = []

    def close(self):
        if getattr(self, "h", None):
            self.lib.tl_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ----------------------------------------------------------- weights
    def load(self, model: Model):
        """Copy a quantized model into the engine. The model must have exactly
        the engine's configuration (layer count, widths, vocabulary): the C
        side reads each array with the sizes the engine was created with, so
        every shape is checked here first and a mismatch raises ValueError."""
        check_model(model, self.cfg)
        cfg = model.cfg
        cos, sin = rope_tables(cfg["max_position_embeddings"], cfg["head_dim"], cfg["rope_theta"])
        keep = [cos, sin]

        def lin(l: Linear) -> LinearView:
            w = np.ascontiguousarray(l.w, dtype=np.int8)
            s = np.ascontiguousarray(l.scale, dtype=np.float64)
            keep.extend([w, s])
            return LinearView(_ptr(w), _ptr(s))

        def arr(a) -> int:
            a = np.ascontiguousarray(a, dtype=np.float32)
            keep.append(a)
            return _ptr(a)

        layers = (LayerView * len(model.layers))()
        for i, ly in enumerate(model.layers):
            layers[i] = LayerView(lin(ly.q), lin(ly.k), lin(ly.v), lin(ly.o), lin(ly.gate), lin(ly.up),
                                  lin(ly.down), arr(ly.input_norm), arr(ly.post_norm))
        view = WeightsView(arr(model.embed), arr(model.final_norm), lin(model.lm_head), layers,
                           _ptr(cos), _ptr(sin))
        check(self.lib.tl_load_weights(self.h, C.byref(view)), "tl_load_weights")

    def init_random(self, seed: int = 0):
        check(self.lib.tl_init_random_weights(self.h, seed), "tl_init_random_weights")

    # ----------------------------------------------------------- runtime
    def generate(self, prompt, max_new_tokens: int, eos_id: int = 0xFFFFFFFF, mode: int = MODE_PREFILL,
                 out_cap: int | None = None, raise_on_error: bool = True):
        """Greedy generation in slot 0. Returns (tokens, status dict)."""
        ids = np.ascontiguousarray(np.asarray(list(prompt), dtype=np.uint32))
        cap = out_cap if out_cap is not None else max(1, max_new_tokens or self.cfg["max_position_embeddings"])
        out = np.zeros(cap, dtype=np.uint32)
        st = RunStatus()
        code = self.lib.tl_generate(self.h, _ptr(ids) if ids.size else None, ids.size, max_new_tokens,
                                    eos_id & 0xFFFFFFFF, mode, _ptr(out), cap, C.byref(st))
        if raise_on_error and code not in (TL_OK,):
            check(code, "tl_generate")
        d = st.as_dict()
        d["return_code"] = code
        return [int(t) for t in out[:st.generated_count]], d

    def generate_batch(self, prompts: np.ndarray, max_new_tokens: int, eos_id: int = 0xFFFFFFFF,
                       out_cap: int | None = None):
        p = np.ascontiguousarray(np.asarray(prompts, dtype=np.uint32))
        n, s = p.shape
        cap = out_cap if out_cap is not None else max(1, max_new_tokens)
        out = np.zeros((n, cap), dtype=np.uint32)
        st = (RunStatus * n)()
        check(self.lib.tl_generate_batch(self.h, n, _ptr(p), s, max_new_tokens, eos_id & 0xFFFFFFFF,
                                         _ptr(out), cap, st), "tl_generate_batch")
        return [[int(t) for t in out[i, :st[i].generated_count]] for i in range(n)], [x.as_dict() for x in st]

    def abort(self):
        check(self.lib.tl_abort(self.h), "tl_abort")

    def prefill_logits(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(list(ids), dtype=np.uint32))
        out = np.zeros(self.cfg["vocab_size"], dtype=np.float32)
        check(self.lib.tl_prefill_logits(self.h, 0, _ptr(ids), ids.size, _ptr(out)), "tl_prefill_logits")
        return out

    def forward_logits(self, ids, hidden: bool = False):
        """float32 logits of every prompt row, [len(ids), vocab] (tl_forward_logits:
        forward_mixed's output, model/tinyllama_gemm_int8.py:437-467). Leaves
        the prompt prefilled in slot 0. ``hidden=True`` returns instead the
        final RMSNorm output [len(ids), hidden] (the LM head's input) and
        skips the LM head."""
        ids = np.ascontiguousarray(np.asarray(list(ids), dtype=np.uint32))
        if hidden:
            out = np.zeros((ids.size, self.cfg["hidden_size"]), dtype=np.float32)
            args = (None, _ptr(out))
        else:
            out = np.zeros((ids.size, self.cfg["vocab_size"]), dtype=np.float32)
            args = (_ptr(out), None)
        check(self.lib.tl_forward_logits(self.h, _ptr(ids) if ids.size else None, ids.size, *args),
              "tl_forward_logits")
        return out

    def _capture(self, capture, S: int, groups: int, windows: bool):
        c = self.cfg
        dims = {"S": S, "D": c["hidden_size"], "Dq": c["num_attention_heads"] * c["head_dim"],
                "Dkv": c["num_key_value_heads"] * c["head_dim"], "F": c["intermediate_size"]}
        if capture is True:
            capture = [n for n, _, k in CAPTURE_FIELDS if k != "HSS"]
        want = set(capture or ())
        unknown = want - {n for n, _, _ in CAPTURE_FIELDS}
        if unknown:
            raise ValueError(f"unknown capture fields {sorted(unknown)}")
        arrays, cap = {}, LayerCapture()
        for name, dt, key in CAPTURE_FIELDS:
            if name not in want:
                continue
            if key == "HSS" and not windows:
                raise ValueError(f"{name}: score windows are captured by decoder_layer only")
            shape = ((groups,) if key == "1" else (c["num_attention_heads"], S, S) if key == "HSS"
                     else (S, dims[key[1:]]))
            arrays[name] = np.zeros(shape, dtype=dt)
            setattr(cap, name, _ptr(arrays[name]))
        return arrays, (C.byref(cap) if want else None), cap

    def decode_layer(self, layer: int, x, slots, positions, capture=None):
        """One decoder layer of a batched decode step on caller-given rows
        (tl_decode_layer): row r of ``x`` [n, hidden] is the token at
        ``positions[r]`` of the sequence in KV slot ``slots[r]``; its K/V row
        is appended there. n >= 16 (the tensor-core decode path). Returns
        (out [n, hidden], capture dict; ``*_input_absmax`` one float per row)."""
        xf = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
        n = xf.shape[0]
        if xf.ndim != 2 or xf.shape[1] != self.cfg["hidden_size"]:
            raise ValueError(f"x must be [n, {self.cfg['hidden_size']}], got {xf.shape}")
        sl = np.ascontiguousarray(np.asarray(slots, dtype=np.uint32))
        ps = np.ascontiguousarray(np.asarray(positions, dtype=np.uint32))
        if sl.shape != (n,) or ps.shape != (n,):
            raise ValueError("slots and positions need one entry per row")
        arrays, ref, _keep = self._capture(capture, n, n, False)
        out = np.zeros_like(xf)
        check(self.lib.tl_decode_layer(self.h, layer, n, _ptr(sl), _ptr(ps), _ptr(xf), _ptr(out), ref),
              "tl_decode_layer")
        return out, arrays

    def decoder_layer(self, layer: int, x, slot: int = 0, capture=None):
        """One decoder layer of this engine on caller-given activations
        (teacher forcing, tl_decoder_layer): ``x`` float32 [S, hidden] is one
        sequence at positions 0..S-1; layer ``layer``'s K/V for those rows go
        into KV slot ``slot``. ``capture`` names the intermediate tensors to
        return (fields of ``CAPTURE_FIELDS``; ``True`` = all but the [H,S,S]
        score and probability windows). Returns (out [S, hidden], dict)."""
        xf = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
        if xf.ndim != 2 or xf.shape[1] != self.cfg["hidden_size"]:
            raise ValueError(f"x must be [S, {self.cfg['hidden_size']}], got {xf.shape}")
        S = xf.shape[0]
        arrays, ref, _keep = self._capture(capture, S, 1, True)
        out = np.zeros_like(xf)
        check(self.lib.tl_decoder_layer(self.h, slot, layer, _ptr(xf), S, _ptr(out), ref), "tl_decoder_layer")
        return out, arrays

    def decode_debug(self, token: int, layer: int, slot: int = 0, logits: bool = False) -> dict:
        """One decode step of ``slot`` fed ``token`` with the debug capture of
        layer ``layer`` (tl_decode_debug, the hardware's debug contract,
        docs/design_decisions.txt B8): a dict of every record field (arrays as
        numpy), plus ``logits`` [vocab] when asked."""
        c = self.cfg
        pos = self.position(slot)
        hkv = c["num_key_value_heads"]
        shapes = {"D": (c["hidden_size"],), "Dq": (c["num_attention_heads"] * c["head_dim"],),
                  "Dkv": (hkv * c["head_dim"],), "Hn": (c["num_attention_heads"], pos + 1),
                  "Hkv64": (hkv, 64), "Hkv": (hkv,)}
        rec, out = DebugRecord(), {}
        for name, dt, key in DEBUG_FIELDS:
            out[name] = np.zeros(shapes[key], dtype=dt)
            setattr(rec, name, _ptr(out[name]))
        lg = np.zeros(c["vocab_size"], np.float32) if logits else None
        check(self.lib.tl_decode_debug(self.h, slot, int(token), layer, C.byref(rec),
                                       _ptr(lg) if lg is not None else None), "tl_decode_debug")
        out.update(position=rec.position, chosen_token=rec.chosen_token,
                   top_ids=np.array(rec.top_ids[:], np.int64), top_logits=np.array(rec.top_logits[:], np.float32),
                   input_absmax=np.array(rec.input_absmax[:], np.float32))
        if lg is not None:
            out["logits"] = lg
        return out

    def decode_logits(self, token: int, slot: int = 0) -> np.ndarray:
        out = np.zeros(self.cfg["vocab_size"], dtype=np.float32)
        check(self.lib.tl_decode_logits(self.h, slot, int(token), _ptr(out)), "tl_decode_logits")
        return out

    def read_kv(self, layer: int, n_pos: int, slot: int = 0):
        """INT8 K/V rows [kv_head][pos][64] and scales of one layer (this
        rank's kv heads on a tensor-parallel engine)."""
        hkv = self.cfg["num_key_value_heads"] // self.tp_world
        k = np.zeros((hkv, n_pos, 64), np.int8)
        v = np.zeros((hkv, n_pos, 64), np.int8)
        ks = np.zeros(hkv, np.float32)
        vs = np.zeros(hkv, np.float32)
        check(self.lib.tl_read_kv(self.h, slot, layer, n_pos, _ptr(k), _ptr(v), _ptr(ks), _ptr(vs)),
              "tl_read_kv")
        return k, v, ks, vs

    def position(self, slot: int = 0) -> int:
        p = C.c_uint32()
        check(self.lib.tl_get_position(self.h, slot, C.byref(p)), "tl_get_position")
        return p.value

    # ------------------------------------------------ device-resident (bench)
    def prefill_batch_device(self, prompts: np.ndarray):
        p = np.ascontiguousarray(np.asarray(prompts, dtype=np.uint32))
        check(self.lib.tl_prefill_batch_device(self.h, p.shape[0], _ptr(p), p.shape[1]),
              "tl_prefill_batch_device")

    def decode_steps_device(self, n_seqs: int, steps: int):
        check(self.lib.tl_decode_steps_device(self.h, n_seqs, steps), "tl_decode_steps_device")

    def decode_rewind(self, n_seqs: int, position: int):
        check(self.lib.tl_decode_rewind(self.h, n_seqs, position), "tl_decode_rewind")

    def synchronize(self):
        check(self.lib.tl_synchronize(self.h), "tl_synchronize")

    def stream_handle(self) -> int:
        return self.lib.tl_engine_stream(self.h) or 0

    def profile_decode_kernels(self, n_seqs: int, iters: int = 44) -> np.ndarray:
        """Average device time (ms) of each decode kernel kind, see
        tl_profile_decode_kernels: [qkv, attn, o, gate_up, down, lm_head,
        norm_quant_rows, quant_rows]."""
        out = np.zeros(8, dtype=np.float32)
        check(self.lib.tl_profile_decode_kernels(self.h, n_seqs, iters, _ptr(out)),
              "tl_profile_decode_kernels")
        return out

    def decode_step_kernel_count(self, n_seqs: int = 1) -> int:
        return int(self.lib.tl_decode_step_kernel_count_rows(self.h, n_seqs))

    def decode_row_groups(self, n_seqs: int) -> int:
        """Concurrent row groups (streams) of a decode step of n_seqs rows."""
        return int(self.lib.tl_decode_row_groups(self.h, n_seqs))


# --------------------------------------------------------------------------
# Operator API (device tensors via torch for buffers; compute in the library)
# --------------------------------------------------------------------------
def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device visible: the operator API runs only on the GPU")
    return torch


def _stream(torch):
    return torch.cuda.current_stream().cuda_stream


def quantize_int8(t: np.ndarray):
    """GPU ``quantize_int8`` (model/tinyllama_gemm_int8.py:36-42): returns
    (int8 array, scale as a Python float)."""
    torch = _torch()
    lib = load_library()
    x = np.ascontiguousarray(np.asarray(t, dtype=np.float32))
    flat = x.reshape(1, -1) if x.ndim != 2 else x
    rows, cols = flat.shape
    if x.ndim != 2:
        rows, cols = 1, x.size
    dx = torch.from_numpy(flat.reshape(rows, cols)).cuda()
    q = torch.empty((rows, cols), dtype=torch.int8, device="cuda")
    am = torch.empty(1, dtype=torch.float32, device="cuda")
    check(lib.tl_quantize_int8(dx.data_ptr(), rows, cols, rows, q.data_ptr(), am.data_ptr(), _stream(torch)),
          "tl_quantize_int8")
    peak = float(am.item())
    scale = 1.0 if peak == 0.0 else peak / 127.0
    return q.cpu().numpy().reshape(x.shape), scale


def quantized_linear(x: np.ndarray, w: np.ndarray, b: np.ndarray | None = None, capture_arrays: bool = False):
    """GPU ``quantized_linear`` (model/tinyllama_gemm_int8.py:59-88): x [S,K]
    float, w [K,N] float quantized per tensor, INT8 GEMM with INT32
    accumulation, dequantized output [S,N] float32."""
    torch = _torch()
    lib = load_library()
    x_fp = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    w_fp = np.asarray(w, dtype=np.float32)
    lw = quantize_weight(w_fp, "tensor")
    m, k = x_fp.shape
    n = w_fp.shape[1]
    if k % 16:
        raise ValueError("K must be a multiple of 16")
    dx = torch.from_numpy(x_fp).cuda()
    wkn = torch.from_numpy(np.ascontiguousarray(lw.w)).cuda()
    wnk = torch.empty((n, k), dtype=torch.int8, device="cuda")
    st = _stream(torch)
    check(lib.tl_transpose_i8(wkn.data_ptr(), wnk.data_ptr(), k, n, st), "tl_transpose_i8")
    ws = torch.from_numpy(lw.scale).cuda()
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda") if capture_arrays else None
    check(lib.tl_quantized_linear(dx.data_ptr(), wnk.data_ptr(), ws.data_ptr(), out.data_ptr(),
                                  acc.data_ptr() if acc is not None else None, m, n, k, st),
          "tl_quantized_linear")
    o = out.cpu().numpy()
    if b is not None:
        o = o + np.asarray(b, dtype=np.float32)
    xq, sx = quantize_int8(x_fp)
    dbg = {"input_scale": np.array([sx], dtype=np.float32),
           "weight_scale": np.array([lw.scale[0]], dtype=np.float32)}
    if capture_arrays:
        dbg.update({"input_fp": x_fp, "input_q": xq, "weight_fp": w_fp, "weight_q": lw.w,
                    "accum_int32": acc.cpu().numpy(), "output_fp": o.astype(np.float32)})
    return o.astype(np.float32), dbg


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """GPU ``rms_norm`` (model/tinyllama.py:45-50), bit-exact with NumPy."""
    torch = _torch()
    lib = load_library()
    xf = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    shp = xf.shape
    x2 = xf.reshape(-1, shp[-1])
    dx = torch.from_numpy(x2).cuda()
    g = torch.from_numpy(np.ascontiguousarray(np.asarray(w, np.float32))).cuda()
    out = torch.empty_like(dx)
    check(lib.tl_rmsnorm(dx.data_ptr(), g.data_ptr(), float(eps), out.data_ptr(), x2.shape[0], x2.shape[1],
                         _stream(torch)), "tl_rmsnorm")
    return out.cpu().numpy().reshape(shp)


_ENGINE_CACHE: "OrderedDict" = OrderedDict()
_ENGINE_CACHE_MAX = 4


def _cached_engine(key, owner, make_model, cfg: dict, max_prefill: int):
    """Engine for a weights object (or a reference layer dict), reused while
    the caller passes the same object: the cache holds a reference to
    ``owner`` so its id cannot be reused while cached. The least recently used
    of more than four engines is closed (each holds device memory)."""
    hit = _ENGINE_CACHE.get(key)
    if hit is not None and hit[0] is owner:
        _ENGINE_CACHE.move_to_end(key)
        return hit[1]
    if hit is not None:
        hit[1].close()
        del _ENGINE_CACHE[key]
    while len(_ENGINE_CACHE) >= _ENGINE_CACHE_MAX:
        _, (_, old) = _ENGINE_CACHE.popitem(last=False)
        old.close()
    model = make_model()
    eng = Engine(model.cfg, max_batch=1, max_prefill_tokens=max_prefill)
    eng.load(model)
    _ENGINE_CACHE[key] = (owner, eng)
    return eng


def forward_mixed(token_ids, weights, cos=None, sin=None, layer_count: int | None = None,
                  quantize_lm_head: bool = True) -> np.ndarray:
    """GPU ``forward_mixed`` (model/tinyllama_gemm_int8.py:437-467) for a
    ``TinyLlamaWeights``-like object: logits of every row, float32 [S, vocab].
    Weights are quantized per tensor, as the reference bridge does on every
    call; attention reads the engine's INT8 KV cache (per-(layer, kv head)
    scales calibrated on the prompt), the one place the engine's numerics
    differ from the reference's float K/V. ``quantize_lm_head=False`` takes
    the final RMSNorm output from the engine and multiplies it by the float
    LM head on the GPU (float32, no TF32), as the reference's float branch
    does. ``cos``/``sin`` are accepted for signature compatibility; the
    engine builds the same float32 tables from the config."""
    cfg = dict(weights.cfg)
    n_layers = cfg["num_hidden_layers"] if layer_count is None else int(layer_count)
    if not 0 < n_layers <= cfg["num_hidden_layers"]:
        raise ValueError(f"--layers must be between 1 and {cfg['num_hidden_layers']}")
    if len(token_ids) > cfg["max_position_embeddings"]:
        raise ValueError(f"Sequence length {len(token_ids)} exceeds "
                         f"max_position_embeddings={cfg['max_position_embeddings']}")
    eng = _cached_engine(("model", id(weights), n_layers), weights,
                         lambda: from_tinyllama_weights(weights, n_layers), cfg, cfg["max_position_embeddings"])
    if quantize_lm_head:
        return eng.forward_logits(token_ids)
    torch = _torch()
    hid = eng.forward_logits(token_ids, hidden=True)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        w = torch.from_numpy(np.ascontiguousarray(np.asarray(weights.lm_head_w(), np.float32))).cuda()
        return (torch.from_numpy(hid).cuda() @ w).cpu().numpy().astype(np.float32)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _linear_debug(capture_arrays, input_fp, input_q, absmax, w_fp, w_q, w_scale, acc, output_fp):
    """``quantized_linear``'s debug dict (model/tinyllama_gemm_int8.py:74-86)."""
    peak = float(absmax[0])
    sx = 1.0 if peak == 0.0 else peak / 127.0
    ws = np.asarray(w_scale, np.float64)
    d = {"input_scale": np.array([sx], dtype=np.float32),
         "weight_scale": (np.array([ws[0]], np.float32) if np.all(ws == ws[0]) else ws.astype(np.float32))}
    if capture_arrays:
        d.update({"input_fp": input_fp, "input_q": input_q, "weight_fp": w_fp, "weight_q": w_q,
                  "accum_int32": acc, "output_fp": output_fp})
    return d


def layer_debug(cap: dict, capture_arrays: bool, weights: dict | None = None, quant: dict | None = None) -> dict:
    """Arrange a :meth:`Engine.decoder_layer` capture as the debug dict of
    ``mixed_precision_decoder_layer`` (model/tinyllama_gemm_int8.py:136-281):
    ``attn``/``ffn`` sub-dicts with one ``quantized_linear`` dict per
    projection plus the ``*_fp`` tensors. ``weights`` (float [in, out] by
    projection name) and ``quant`` (Linear by name) fill ``weight_fp`` /
    ``weight_q`` / ``weight_scale`` when given."""
    weights, quant = weights or {}, quant or {}

    def lin(name, inp, inq, am, acc, out):
        q = quant.get(name)
        return _linear_debug(capture_arrays, inp, inq, am, weights.get(name),
                             None if q is None else q.w, [1.0] if q is None else q.scale, acc, out)

    attn = {
        "q_proj": lin("q", cap["attn_input"], cap["qkv_input_q"], cap["qkv_input_absmax"], cap["q_acc"], cap["q_proj"]),
        "k_proj": lin("k", cap["attn_input"], cap["qkv_input_q"], cap["qkv_input_absmax"], cap["k_acc"], cap["k_proj"]),
        "v_proj": lin("v", cap["attn_input"], cap["qkv_input_q"], cap["qkv_input_absmax"], cap["v_acc"], cap["v_proj"]),
        "o_proj": lin("o", cap["attended"], cap["o_input_q"], cap["o_input_absmax"], cap["o_acc"], cap["o_proj"]),
        "q_proj_fp": cap["q_proj"], "k_proj_fp": cap["k_proj"], "v_proj_fp": cap["v_proj"],
    }
    ffn = {
        "gate_proj": lin("gate", cap["ffn_input"], cap["gate_up_input_q"], cap["gate_up_input_absmax"],
                         cap["gate_acc"], cap["gate_proj"]),
        "up_proj": lin("up", cap["ffn_input"], cap["gate_up_input_q"], cap["gate_up_input_absmax"],
                       cap["up_acc"], cap["up_proj"]),
        "down_proj": lin("down", cap["hidden"], cap["down_input_q"], cap["down_input_absmax"], cap["down_acc"],
                         cap["down_proj"]),
        "gate_proj_fp": cap["gate_proj"], "up_proj_fp": cap["up_proj"], "hidden_fp": cap["hidden"],
    }
    if capture_arrays:
        attn.update({"scores_fp": cap.get("scores"), "weights_fp": cap.get("probs"),
                     "attended_fp": cap["attended"], "out_fp": cap["o_proj"]})
        ffn["out_fp"] = cap["down_proj"]
        attn = {k: v for k, v in attn.items() if v is not None}
    return {"attn_input_fp": cap["attn_input"], "x_after_attn_fp": cap["x_after_attn"],
            "ffn_input_fp": cap["ffn_input"], "attn": attn, "ffn": ffn}


def mixed_precision_decoder_layer(x, layer: dict, cfg: dict, cos=None, sin=None, capture_arrays: bool = False):
    """GPU ``mixed_precision_decoder_layer`` (model/tinyllama_gemm_int8.py:256-281).

    ``layer`` is the reference's layer dict (model/tinyllama.py:249-267:
    float ``q_w`` .. ``down_w`` stored [in, out], ``*_b`` biases, the two
    norm gains); ``x`` float32 [S, hidden] is one sequence at positions
    0..S-1. The weights are quantized per tensor (the bridge's per-call rule,
    :69) and the layer runs on the engine's prefill kernels; K and V go
    through the engine's INT8 cache before attention. Returns ``(out,
    debug)`` with the reference's debug keys; ``capture_arrays`` adds the
    per-projection arrays (``input_q``, ``accum_int32``, ...), the [H, S, S]
    score and probability windows and the block outputs. Biases are not
    supported (TinyLlama has none)."""
    for b in ("q_b", "k_b", "v_b", "o_b", "gate_b", "up_b", "down_b"):
        if layer.get(b) is not None:
            raise NotImplementedError(f"projection biases are not supported by the engine ({b})")
    xf = np.asarray(x, dtype=np.float32)
    c = {k: cfg[k] for k in ("hidden_size", "intermediate_size", "num_attention_heads", "num_key_value_heads",
                             "head_dim", "max_position_embeddings", "rms_norm_eps", "rope_theta")}
    c.update(num_hidden_layers=1, vocab_size=16)  # the layer engine never uses the embedding or LM head
    if xf.shape[0] > c["max_position_embeddings"]:
        raise ValueError(f"Sequence length {xf.shape[0]} exceeds max_position_embeddings={c['max_position_embeddings']}")

    def make_model():
        quant = {p: quantize_weight(layer[f"{p}_w"], "tensor") for p in _NPZ_PROJ}
        ly = Layer(*(quant[p] for p in _NPZ_PROJ), input_norm=np.asarray(layer["input_norm_w"], np.float32),
                   post_norm=np.asarray(layer["post_norm_w"], np.float32))
        d = c["hidden_size"]
        m = Model(dict(c), np.zeros((16, d), np.float32), np.ones(d, np.float32),
                  Linear(np.zeros((d, 16), np.int8), np.ones(16)), [ly])
        return m

    eng = _cached_engine(("layer", id(layer)), layer, make_model, c, c["max_position_embeddings"])
    want = [n for n, _, k in CAPTURE_FIELDS if capture_arrays or k != "HSS"]
    out, cap = eng.decoder_layer(0, xf, capture=want)
    quant = {p: quantize_weight(layer[f"{p}_w"], "tensor") for p in _NPZ_PROJ} if capture_arrays else None
    wfp = {p: np.asarray(layer[f"{p}_w"], np.float32) for p in _NPZ_PROJ} if capture_arrays else None
    debug = layer_debug(cap, capture_arrays, wfp, quant)
    if capture_arrays:
        debug["layer_out_fp"] = out
    return out, debug


# --------------------------------------------------------------------------
# Contract mode: the hardware's Q16.16 wrappers (host arrays in and out)
# --------------------------------------------------------------------------
def _dev(torch, a, dtype):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=dtype))).cuda()


def contract_rmsnorm(x_q, in_scale_q16: int, gamma_q16, eps: float, out_scale_q16: int):
    """RMSNorm wrapper (rtl/nonlinear/rmsnorm_wrapper.sv): INT8 rows [R, D] ->
    (y_q16 int32, y_q int8), see tl_contract_rmsnorm."""
    torch = _torch()
    lib = load_library()
    x = _dev(torch, x_q, np.int8)
    rows, cols = x.shape
    yq = torch.empty_like(x)
    y16 = torch.empty((rows, cols), dtype=torch.int32, device="cuda")
    g = _dev(torch, gamma_q16, np.int32)  # held: a temporary's memory would be reused before the launch
    check(lib.tl_contract_rmsnorm(x.data_ptr(), rows, cols, int(in_scale_q16), g.data_ptr(), float(eps),
                                  int(out_scale_q16), yq.data_ptr(), y16.data_ptr(), _stream(torch)),
          "tl_contract_rmsnorm")
    return y16.cpu().numpy(), yq.cpu().numpy()


def contract_silu(x_q, in_scale_q16: int, out_scale_q16: int):
    """SiLU wrapper (rtl/nonlinear/silu_wrapper.sv): -> (y_q16, y_q)."""
    torch = _torch()
    lib = load_library()
    x = _dev(torch, x_q, np.int8)
    yq = torch.empty_like(x)
    y16 = torch.empty(x.shape, dtype=torch.int32, device="cuda")
    check(lib.tl_contract_silu(x.data_ptr(), x.numel(), int(in_scale_q16), int(out_scale_q16), yq.data_ptr(),
                               y16.data_ptr(), _stream(torch)), "tl_contract_silu")
    return y16.cpu().numpy(), yq.cpu().numpy()


def contract_softmax(scores, score_scale_q16: int):
    """Softmax wrapper (rtl/nonlinear/softmax_wrapper.sv): INT32 scores
    [R, C <= 128] -> (prob_q16, prob_q) with the 1/127 probability scale."""
    torch = _torch()
    lib = load_library()
    sc = _dev(torch, scores, np.int32)
    rows, cols = sc.shape
    pq = torch.empty((rows, cols), dtype=torch.int8, device="cuda")
    p16 = torch.empty((rows, cols), dtype=torch.int32, device="cuda")
    check(lib.tl_contract_softmax(sc.data_ptr(), rows, cols, int(score_scale_q16), pq.data_ptr(), p16.data_ptr(),
                                  _stream(torch)), "tl_contract_softmax")
    return p16.cpu().numpy(), pq.cpu().numpy()


def contract_rope(x_q, cos_q16, sin_q16):
    """Q16.16 RoPE of INT8 rows [R, 64] with per-row tables (rope_unit.sv)."""
    torch = _torch()
    lib = load_library()
    x = _dev(torch, x_q, np.int8)
    out = torch.empty_like(x)
    cs, sn = _dev(torch, cos_q16, np.int32), _dev(torch, sin_q16, np.int32)  # held until the launch
    check(lib.tl_contract_rope(x.data_ptr(), cs.data_ptr(), sn.data_ptr(), x.shape[0], out.data_ptr(),
                               _stream(torch)), "tl_contract_rope")
    return out.cpu().numpy()


def residual_add_i32(residual_q16, update_q16):
    """Unsaturated INT32 residual add (residual_add.sv:92-96)."""
    torch = _torch()
    lib = load_library()
    a, b = _dev(torch, residual_q16, np.int32), _dev(torch, update_q16, np.int32)
    out = torch.empty_like(a)
    check(lib.tl_residual_add_i32(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), _stream(torch)),
          "tl_residual_add_i32")
    return out.cpu().numpy()
