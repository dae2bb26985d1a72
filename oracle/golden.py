"""NumPy restatement of the reference INT8 bridge golden model.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Every function here restates one block of the reference's Python golden model
and names the reference lines it follows. The arithmetic is kept operation for
operation (same NumPy dtypes, same scalar promotion rules) because the point of
this module is to be bit-identical to the reference on the same inputs; the
fixture tests in ``tests/test_oracle_golden.py`` check exactly that.

Numerics that the CUDA engine has to reproduce, and that are easy to get wrong:

* ``quantize_int8``: the scale is a Python float (float64) ``max|t| / 127``;
  the division ``t / scale`` is done in float32 against ``float32(scale)``
  (NumPy 2 weak-scalar promotion), then rounded half-to-even.
* ``dequantize_int32``: ``float32(acc) * float32(s_x * s_w)`` where the product
  of the two scales is formed in float64 first.
* ``rms_norm``: the mean of squares is NumPy's float32 pairwise sum
  (restated in :func:`pairwise_sum_f32`) divided by the row length.
* attention: ``attn_scale`` is a NumPy float64 scalar, so scores, softmax and
  the weighted sum run in float64 in the reference.
"""

from __future__ import annotations

import numpy as np

MASK_FILL = -1e9  # model/tinyllama_gemm_int8.py:159 (scores[:, ~mask] = -1e9)


# ----------------------------------------------------------------------------
# Quantization primitives
# ----------------------------------------------------------------------------
def quantize_int8(tensor: np.ndarray) -> tuple[np.ndarray, float]:
    """Symmetric per-tensor INT8 quantization.

    Follows ``quantize_int8`` in model/tinyllama_gemm_int8.py:36-42: scale is
    max|t|/127 as a Python float (1.0 for an all-zero tensor), values are
    rounded half-to-even after a float32 division and clipped to [-127, 127].
    """
    t = np.asarray(tensor, dtype=np.float32)
    peak = float(np.max(np.abs(t))) if t.size else 0.0
    scale = 1.0 if peak == 0.0 else peak / 127.0
    q = np.clip(np.round(t / scale), -127, 127).astype(np.int8)
    return q, scale


def quantize_with_scale(tensor: np.ndarray, scale: float) -> np.ndarray:
    """Quantize with a fixed (e.g. frozen KV-cache) scale, same rounding rule
    as :func:`quantize_int8` (model/tinyllama_gemm_int8.py:40-41)."""
    t = np.asarray(tensor, dtype=np.float32)
    return np.clip(np.round(t / scale), -127, 127).astype(np.int8)


def dequantize_int32(acc: np.ndarray, input_scale, weight_scale) -> np.ndarray:
    """``float32(acc) * float32(s_x * s_w)``.

    Follows model/tinyllama_gemm_int8.py:45-46. ``weight_scale`` may be a
    Python float (reference: per-tensor) or a float64 vector over output
    channels (engine: per-output-channel); the scale product is formed in
    float64 and rounded to float32 once per channel in both cases.
    """
    combined = np.asarray(np.float64(input_scale) * np.asarray(weight_scale, dtype=np.float64))
    return acc.astype(np.float32) * combined.astype(np.float32)


def int8_matmul(a_q: np.ndarray, b_q: np.ndarray) -> np.ndarray:
    """Exact INT8 x INT8 -> INT32 matmul (a [M,K] @ b [K,N]).

    The reference computes ``x_q.astype(int32) @ w_q.astype(int32)``
    (model/tinyllama_gemm_int8.py:70). Every partial sum here is an integer of
    magnitude <= 127*127*K < 2**53, so a float64 BLAS product is exact and
    gives the identical INT32 result much faster.
    """
    prod = np.asarray(a_q, dtype=np.float64) @ np.asarray(b_q, dtype=np.float64)
    return prod.astype(np.int32)


class ExactMatmul:
    """Exact INT8 x INT8 -> INT32 matmul for large models, faster than
    :func:`int8_matmul` when the same weight matrices are used many times.

    Each weight ``b_q`` [K, N] is converted once to float32 (kept while this
    object lives) and the product is formed over K-chunks of at most 1024:
    within a chunk every product and every partial sum is an integer of
    magnitude <= 1024 * 127 * 127 < 2**24, so float32 BLAS is exact in any
    summation order; the chunk results are summed in float64 (exact) and
    returned as INT32, identical to ``x_q.astype(int32) @ w_q.astype(int32)``
    (model/tinyllama_gemm_int8.py:70)."""

    CHUNK = 1024

    def __init__(self):
        self._cache: dict = {}

    def _chunks(self, b_q: np.ndarray):
        hit = self._cache.get(id(b_q))
        if hit is not None and hit[0] is b_q:
            return hit[1]
        k = b_q.shape[0]
        parts = [np.asarray(b_q[i:i + self.CHUNK], dtype=np.float32) for i in range(0, k, self.CHUNK)]
        self._cache[id(b_q)] = (b_q, parts)
        return parts

    def __call__(self, a_q: np.ndarray, b_q: np.ndarray) -> np.ndarray:
        parts = self._chunks(b_q)
        a = np.asarray(a_q, dtype=np.float32)
        acc = None
        for i, bp in enumerate(parts):
            r = (a[:, i * self.CHUNK:i * self.CHUNK + bp.shape[0]] @ bp).astype(np.float64)
            acc = r if acc is None else acc + r
        return acc.astype(np.int32)


def int8_matmul_reference_path(a_q: np.ndarray, b_q: np.ndarray) -> np.ndarray:
    """The reference's own INT32 NumPy matmul (non-BLAS, single thread),
    model/tinyllama_gemm_int8.py:70. Used only to time the CPU baseline."""
    return a_q.astype(np.int32) @ b_q.astype(np.int32)


def quantized_linear(x: np.ndarray, w: np.ndarray, b: np.ndarray | None = None,
                     matmul=int8_matmul) -> tuple[np.ndarray, dict]:
    """Reference ``quantized_linear`` with float weights quantized per tensor
    on every call (model/tinyllama_gemm_int8.py:59-88). Returns the float32
    output and the debug dict keys the reference uses."""
    x_fp = np.asarray(x, dtype=np.float32)
    w_fp = np.asarray(w, dtype=np.float32)
    x_q, sx = quantize_int8(x_fp)
    w_q, sw = quantize_int8(w_fp)
    acc = matmul(x_q, w_q)
    out = dequantize_int32(acc, sx, sw)
    if b is not None:
        out = out + np.asarray(b, dtype=np.float32)
    dbg = {"input_q": x_q, "weight_q": w_q, "accum_int32": acc,
           "input_scale": np.array([sx], dtype=np.float32),
           "weight_scale": np.array([sw], dtype=np.float32)}
    return out.astype(np.float32), dbg


def linear_q(x: np.ndarray, w_q: np.ndarray, w_scale: np.ndarray,
             matmul=int8_matmul) -> tuple[np.ndarray, np.ndarray, float, np.ndarray]:
    """``quantized_linear`` with pre-quantized weights (int8 [K,N] plus a
    float64 scale per output channel). With a per-tensor weight quantization
    broadcast over N this is bit-identical to :func:`quantized_linear`.

    Returns (out fp32, x_q, s_x, acc int32)."""
    x_q, sx = quantize_int8(x)
    acc = matmul(x_q, w_q)
    return dequantize_int32(acc, sx, w_scale), x_q, sx, acc


# ----------------------------------------------------------------------------
# Higher-precision blocks (model/tinyllama.py)
# ----------------------------------------------------------------------------
def pairwise_sum_f32(v: np.ndarray) -> np.float32:
    """NumPy's float32 add-reduce order for one contiguous row.

    Leaves of <= 128 elements use eight running float32 sums over a stride of
    8, folded as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) plus a scalar tail; longer
    runs split at n/2 rounded down to a multiple of 8. ``np.mean(x*x, -1)`` in
    ``rms_norm`` (model/tinyllama.py:48) reduces in this order, and the CUDA
    RMSNorm follows the same tree, which makes it bit-exact.
    """
    v = np.asarray(v, dtype=np.float32)
    n = v.shape[0]
    if n < 8:
        acc = np.float32(0.0)
        for e in v:
            acc = np.float32(acc + e)
        return acc
    if n <= 128:
        lanes = v[:8].copy()
        full = n - (n % 8)
        for base in range(8, full, 8):
            lanes = (lanes + v[base:base + 8]).astype(np.float32)
        acc = np.float32((np.float32(lanes[0] + lanes[1]) + np.float32(lanes[2] + lanes[3]))
                         + (np.float32(lanes[4] + lanes[5]) + np.float32(lanes[6] + lanes[7])))
        for e in v[full:]:
            acc = np.float32(acc + e)
        return acc
    half = n // 2
    half -= half % 8
    return np.float32(pairwise_sum_f32(v[:half]) + pairwise_sum_f32(v[half:]))


def rms_norm(x: np.ndarray, gamma: np.ndarray, eps: float) -> np.ndarray:
    """x * (1/sqrt(mean(x^2) + eps)) * gamma in float32 (model/tinyllama.py:45-50)."""
    xf = np.asarray(x, dtype=np.float32)
    g = np.asarray(gamma, dtype=np.float32)
    ms = np.mean(xf * xf, axis=-1, keepdims=True)
    inv = 1.0 / np.sqrt(ms + eps)
    return xf * inv * g


def build_rope_cache(n_pos: int, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """float32 cos/sin tables [n_pos, head_dim] (model/tinyllama.py:59-66).
    The two halves of the last axis repeat the same frequencies."""
    exponent = np.arange(0, head_dim, 2, dtype=np.float32) / head_dim
    inv_freq = 1.0 / (theta ** exponent)
    ang = np.outer(np.arange(n_pos, dtype=np.float32), inv_freq)
    ang = np.concatenate([ang, ang], axis=-1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """[-x2, x1] over the last axis (model/tinyllama.py:69-71)."""
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def rope(x: np.ndarray, cos_rows: np.ndarray, sin_rows: np.ndarray) -> np.ndarray:
    """x*cos + rotate_half(x)*sin, no fused multiply-add (model/tinyllama.py:74-80).
    ``x`` is [heads, S, head_dim]; ``cos_rows``/``sin_rows`` are [S, head_dim]."""
    return (x * cos_rows[np.newaxis]) + (rotate_half(x) * sin_rows[np.newaxis])


def causal_mask(n: int) -> np.ndarray:
    """Lower-triangular boolean mask (model/tinyllama.py:90-91)."""
    return np.tril(np.ones((n, n), dtype=bool))


def repeat_kv(x: np.ndarray, groups: int) -> np.ndarray:
    """GQA fan-out along the head axis (model/tinyllama.py:94-97)."""
    return x if groups == 1 else np.repeat(x, groups, axis=0)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """Max-shifted softmax (model/tinyllama.py:100-103)."""
    e = np.exp(x - np.max(x, axis=axis, keepdims=True))
    return e / np.sum(e, axis=axis, keepdims=True)


def silu(x: np.ndarray) -> np.ndarray:
    """x / (1 + exp(-clip(x, -60, 60))) in float32 (model/tinyllama.py:159-161)."""
    xf = np.asarray(x, dtype=np.float32)
    return xf / (1.0 + np.exp(-np.clip(xf, -60.0, 60.0)))


def attention_core(q_heads: np.ndarray, k_heads: np.ndarray, v_heads: np.ndarray,
                   groups: int, attn_scale, causal: bool) -> np.ndarray:
    """Scores, mask, softmax and weighted sum over GQA heads.

    Follows model/tinyllama_gemm_int8.py:156-163. ``q_heads`` is [H, Sq, hd],
    ``k_heads``/``v_heads`` are [Hkv, Skv, hd]. ``attn_scale`` is the NumPy
    float64 ``1/sqrt(head_dim)`` of model/tinyllama.py:221, which promotes the
    scores and everything after them to float64. Returns [Sq, H*hd]."""
    k_rep = repeat_kv(k_heads, groups)
    v_rep = repeat_kv(v_heads, groups)
    scores = (q_heads @ k_rep.transpose(0, 2, 1)) * attn_scale
    if causal:
        scores[:, ~causal_mask(scores.shape[-1])] = MASK_FILL
    probs = softmax(scores, axis=-1)
    out = probs @ v_rep
    n_heads, sq, hd = q_heads.shape
    return out.transpose(1, 0, 2).reshape(sq, n_heads * hd)


def attention_core_f32(q_heads: np.ndarray, k_heads: np.ndarray, v_heads: np.ndarray,
                       groups: int, attn_scale, causal: bool) -> np.ndarray:
    """:func:`attention_core` with every step in float32 instead of the
    reference's float64 (scores, mask, softmax, weighted sum). Not the
    reference's numerics: it exists to measure how far the reference's own
    INT8 pipeline moves when only the attention arithmetic changes by
    float32 rounding (the sensitivity that end-to-end tolerances are set
    against)."""
    q = np.asarray(q_heads, np.float32)
    k_rep = repeat_kv(np.asarray(k_heads, np.float32), groups)
    v_rep = repeat_kv(np.asarray(v_heads, np.float32), groups)
    scores = (q @ k_rep.transpose(0, 2, 1)) * np.float32(attn_scale)
    if causal:
        scores[:, ~causal_mask(scores.shape[-1])] = np.float32(MASK_FILL)
    e = np.exp(scores - np.max(scores, axis=-1, keepdims=True))
    probs = e / np.sum(e, axis=-1, keepdims=True)
    out = probs @ v_rep
    n_heads, sq, hd = q.shape
    return out.transpose(1, 0, 2).reshape(sq, n_heads * hd)


def attention_core_noisy(seed: int, rel: float = 2e-6):
    """:func:`attention_core` whose output is perturbed by Gaussian noise of
    ``rel`` x max|output| (fresh noise per call, seeded). Not the reference's
    numerics: it models any implementation whose attention is within ``rel``
    of the float64 reference (2e-6 is the accuracy the decode attention
    tests hold the CUDA kernels to), to measure how far that moves the
    reference's own INT8 pipeline end to end."""
    rng = np.random.default_rng(seed)

    def core(q_heads, k_heads, v_heads, groups, attn_scale, causal):
        out = attention_core(q_heads, k_heads, v_heads, groups, attn_scale, causal)
        peak = float(np.max(np.abs(out))) if out.size else 0.0
        return out + rel * peak * rng.standard_normal(out.shape)

    return core


# ----------------------------------------------------------------------------
# Decoder layer and full forward, reference semantics (no KV cache)
# ----------------------------------------------------------------------------
def split_heads(t: np.ndarray, n_heads: int, head_dim: int) -> np.ndarray:
    """[S, n*hd] -> [n, S, hd] (model/tinyllama_gemm_int8.py:150-152)."""
    s = t.shape[0]
    return t.reshape(s, n_heads, head_dim).transpose(1, 0, 2)


def decoder_layer_mixed(x: np.ndarray, layer, cfg: dict, cos: np.ndarray, sin: np.ndarray,
                        matmul=int8_matmul) -> np.ndarray:
    """One mixed-precision decoder layer on all S rows, no cache.

    Follows ``mixed_precision_decoder_layer`` (model/tinyllama_gemm_int8.py:256-281)
    with ``mixed_precision_self_attention`` (:136-182) and
    ``mixed_precision_feed_forward`` (:205-225). ``layer`` holds pre-quantized
    weights (``oracle.weights.QLayer``)."""
    s = x.shape[0]
    eps = cfg["rms_norm_eps"]
    h = rms_norm(x, layer.input_norm, eps)
    q, _, _, _ = linear_q(h, layer.q.w_q, layer.q.scale, matmul)
    k, _, _, _ = linear_q(h, layer.k.w_q, layer.k.scale, matmul)
    v, _, _, _ = linear_q(h, layer.v.w_q, layer.v.scale, matmul)
    qh = split_heads(q, cfg["num_attention_heads"], cfg["head_dim"])
    kh = split_heads(k, cfg["num_key_value_heads"], cfg["head_dim"])
    vh = split_heads(v, cfg["num_key_value_heads"], cfg["head_dim"])
    qh = rope(qh, cos[:s], sin[:s])
    kh = rope(kh, cos[:s], sin[:s])
    att = attention_core(qh, kh, vh, cfg["num_key_value_groups"], cfg["attn_scale"], True)
    o, _, _, _ = linear_q(att, layer.o.w_q, layer.o.scale, matmul)
    x1 = x + o
    h2 = rms_norm(x1, layer.post_norm, eps)
    g, _, _, _ = linear_q(h2, layer.gate.w_q, layer.gate.scale, matmul)
    u, _, _, _ = linear_q(h2, layer.up.w_q, layer.up.scale, matmul)
    hid = silu(g) * u
    d, _, _, _ = linear_q(hid, layer.down.w_q, layer.down.scale, matmul)
    return (x1 + d).astype(np.float32)


def reference_decoder_layer(x: np.ndarray, layer: dict, cfg: dict, cos: np.ndarray,
                            sin: np.ndarray) -> np.ndarray:
    """The float32 decoder layer the reference compares the INT8 path with
    (``reference_decoder_layer``, model/tinyllama_gemm_int8.py:228-253, over
    ``reference_self_attention`` :91-133 and ``reference_feed_forward``
    :185-202): the same blocks with ``x @ W`` float matmuls. ``layer`` is a
    reference-schema dict of float [in, out] weights (``q_w`` ..) and norm
    gains (``input_norm_w``, ``post_norm_w``); no biases."""
    s = x.shape[0]
    eps = cfg["rms_norm_eps"]
    f32 = lambda a: np.asarray(a, dtype=np.float32)
    h = rms_norm(x, layer["input_norm_w"], eps)
    q = (h @ f32(layer["q_w"])).astype(np.float32)
    k = (h @ f32(layer["k_w"])).astype(np.float32)
    v = (h @ f32(layer["v_w"])).astype(np.float32)
    qh = rope(split_heads(q, cfg["num_attention_heads"], cfg["head_dim"]), cos[:s], sin[:s])
    kh = rope(split_heads(k, cfg["num_key_value_heads"], cfg["head_dim"]), cos[:s], sin[:s])
    vh = split_heads(v, cfg["num_key_value_heads"], cfg["head_dim"])
    att = attention_core(qh, kh, vh, cfg["num_key_value_groups"], cfg["attn_scale"], True)
    o = (f32(att) @ f32(layer["o_w"])).astype(np.float32)
    x1 = x + o
    h2 = rms_norm(x1, layer["post_norm_w"], eps)
    g = (h2 @ f32(layer["gate_w"])).astype(np.float32)
    u = (h2 @ f32(layer["up_w"])).astype(np.float32)
    d = ((silu(g) * u) @ f32(layer["down_w"])).astype(np.float32)
    return (x1 + d).astype(np.float32)


def forward_mixed(token_ids, model, cos: np.ndarray, sin: np.ndarray,
                  n_layers: int | None = None, matmul=int8_matmul) -> np.ndarray:
    """Logits for every row, recomputing the whole prefix
    (model/tinyllama_gemm_int8.py:437-467, with ``quantize_lm_head=True``)."""
    cfg = model.cfg
    if len(token_ids) > cfg["max_position_embeddings"]:
        raise ValueError("sequence longer than max_position_embeddings")
    x = model.embed[np.asarray(token_ids)].astype(np.float32)
    n = len(model.layers) if n_layers is None else n_layers
    for li in range(n):
        x = decoder_layer_mixed(x, model.layers[li], cfg, cos, sin, matmul)
    x = rms_norm(x, model.final_norm, cfg["rms_norm_eps"])
    logits, _, _, _ = linear_q(x, model.lm_head.w_q, model.lm_head.scale, matmul)
    return logits.astype(np.float32)


def argmax_first(row: np.ndarray) -> int:
    """Greedy token: the first (lowest id) maximum, as ``np.argmax`` in
    model/tinyllama_gemm_int8.py:671 and the RTL tie rule in
    rtl/compute/argmax_reduction.sv:47-58."""
    return int(np.argmax(row))


def generate_recompute(prompt, model, cos, sin, max_new_tokens: int, eos_id=None,
                       matmul=int8_matmul) -> list[int]:
    """Greedy generation that recomputes the prefix each step
    (``run_generate``, model/tinyllama_gemm_int8.py:629-685)."""
    ids = list(prompt)
    out = []
    for _ in range(max_new_tokens):
        tok = argmax_first(forward_mixed(ids, model, cos, sin, matmul=matmul)[-1])
        ids.append(tok)
        out.append(tok)
        if eos_id is not None and tok == eos_id:
            break
    return out
