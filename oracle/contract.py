"""Fixed-point and control contracts pinned by the reference RTL and exporter.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

These are the integer rules of the hardware path (benchmark config 1's
requantize epilogue, the Q16.16 RoPE variant, the argmax tie rule, the stop
priority and the KV-cache address map). Each function restates one reference
rule and names its lines.
"""

from __future__ import annotations

import numpy as np

Q16_FRAC = 16
Q16_ONE = 1 << Q16_FRAC
Q16_HALF = 1 << (Q16_FRAC - 1)


def q16_16_from_float(value: float) -> np.uint32:
    """Unsigned Q16.16 with negative inputs clamped to 0, Python ``round``
    (half to even) on value * 65536, saturated to 32 bits
    (model/export_fpga_vectors.py:152-155)."""
    scaled = int(round(max(0.0, float(value)) * float(Q16_ONE)))
    return np.uint32(min(max(scaled, 0), 0xFFFFFFFF))


def q16_16_signed_from_float(value: float) -> np.int32:
    """Signed Q16.16, saturated to int32 (model/export_fpga_vectors.py:158-161)."""
    scaled = int(round(float(value) * float(Q16_ONE)))
    return np.int32(min(max(scaled, -(1 << 31)), (1 << 31) - 1))


def requant_multiplier_q16(input_scale: float, weight_scale: float, output_scale: float) -> np.uint32:
    """(s_in * s_w) / s_out as Q16.16 (model/export_fpga_vectors.py:542-545)."""
    return q16_16_from_float((input_scale * weight_scale) / float(output_scale))


def _round_shift16_half_even(mag: np.ndarray) -> np.ndarray:
    """Magnitude >> 16 with round-half-to-even on the 16 dropped bits."""
    quot = mag >> Q16_FRAC
    rem = mag & (Q16_ONE - 1)
    up = (rem > Q16_HALF) | ((rem == Q16_HALF) & ((quot & 1) == 1))
    return quot + up.astype(np.int64)


def requantize_q16(acc: np.ndarray, scale_q16, nonnegative_only: bool = False) -> np.ndarray:
    """INT32 accumulator x unsigned Q16.16 multiplier -> INT8.

    ``requantize_scalar`` of rtl/compute/requantize_unit.sv:39-93: 64-bit
    signed product, magnitude shifted right by 16 with round-half-to-even,
    sign restored, clamped to [-127, 127] (or to [0, 127] when
    ``nonnegative_only``). ``scale_q16`` broadcasts against ``acc`` (per
    tensor, or one entry per output column)."""
    a = np.asarray(acc, dtype=np.int64)
    s = np.asarray(scale_q16, dtype=np.int64)
    prod = a * s
    mag = np.abs(prod)
    r = _round_shift16_half_even(mag)
    signed = np.where(prod < 0, -r, r)
    lo = 0 if nonnegative_only else -127
    return np.clip(signed, lo, 127).astype(np.int8)


def round_q16_16_sum_to_int8(total: np.ndarray) -> np.ndarray:
    """Signed Q16.16 sum -> INT8, round-half-to-even, clamp +-127
    (model/export_fpga_vectors.py:684-697; same rounding as rope_unit.sv:73-127)."""
    t = np.asarray(total, dtype=np.int64)
    r = _round_shift16_half_even(np.abs(t))
    return np.clip(np.where(t < 0, -r, r), -127, 127).astype(np.int8)


def rope_int8(x_q: np.ndarray, cos_q16: np.ndarray, sin_q16: np.ndarray) -> np.ndarray:
    """Q16.16 RoPE on INT8 rows [T, 64] with per-row tables [T, 64]
    (model/export_fpga_vectors.py:700-732): lower half x*cos - x[i+32]*sin,
    upper half x*cos + x[i-32]*sin, then :func:`round_q16_16_sum_to_int8`."""
    x = np.asarray(x_q, dtype=np.int64)
    c = np.asarray(cos_q16, dtype=np.int64)
    s = np.asarray(sin_q16, dtype=np.int64)
    half = x.shape[-1] // 2
    pair = np.concatenate([x[..., half:], x[..., :half]], axis=-1)
    sign = np.concatenate([-np.ones(half, np.int64), np.ones(half, np.int64)])
    return round_q16_16_sum_to_int8(x * c + sign * pair * s)


def argmax_lowest_id(logits: np.ndarray) -> int:
    """Largest logit, ties broken toward the lower token id
    (``candidate_better``, rtl/compute/argmax_reduction.sv:47-58)."""
    return int(np.argmax(np.asarray(logits)))


def stop_decision(abort: bool, token_valid: bool, token: int, count: int, max_new: int,
                  eos: int) -> tuple[bool, int]:
    """Stop priority HOST_ABORT(3) > EOS(1) > MAX_TOKENS(2); ``count`` is the
    number of tokens emitted before this one and ``max_new == 0`` means no
    limit (rtl/control/stop_condition_unit.sv:18-37)."""
    if abort:
        return True, 3
    if token_valid and token == eos:
        return True, 1
    if token_valid and max_new != 0 and count + 1 >= max_new:
        return True, 2
    return False, 0


def kv_row_address(base: int, layer: int, kv_head: int, token: int, n_kv_heads: int = 4,
                   max_pos: int = 2048, row_bytes: int = 64) -> int:
    """Byte address of one cached K or V row, layout [layer][kv_head][token][64]
    (rtl/memory/kv_cache_manager.sv:43-44)."""
    return base + (((layer * n_kv_heads) + kv_head) * max_pos + token) * row_bytes


def scale_index(tensor_slot: int, layer: int, kv_head: int, n_layers: int = 22,
                n_kv_heads: int = 4) -> int:
    """Scale-metadata slot ((tensor*22 + layer)*4 + kv_head)
    (rtl/memory/scale_metadata_store.sv:42-52)."""
    return ((tensor_slot * n_layers) + layer) * n_kv_heads + kv_head


def status_word(busy: bool, done: bool, error: bool, stop_valid: bool, stop_reason: int,
                error_code: int) -> int:
    """Packed STATUS register: bit0 busy, bit1 done, bit2 error, bit3
    stop_valid, bits[6:4] stop_reason, bits[11:8] error_code
    (rtl/common/tinyllama_pkg.sv:159-166)."""
    return (int(busy) | (int(done) << 1) | (int(error) << 2) | (int(stop_valid) << 3)
            | ((stop_reason & 0x7) << 4) | ((error_code & 0xF) << 8))


# ----------------------------------------------------------------------------
# Fixed-point wrapper chain of the nonlinear blocks (contract mode)
# ----------------------------------------------------------------------------
def float_from_q16_16(raw) -> np.ndarray:
    """float32(raw / 65536) with the division in float64
    (model/export_fpga_vectors.py:191-192)."""
    return (np.asarray(raw, dtype=np.int64).astype(np.float64) / float(Q16_ONE)).astype(np.float32)


def q16_16_signed_array(values) -> np.ndarray:
    """Elementwise :func:`q16_16_signed_from_float` (Python round, half to
    even, of value * 65536; saturated to int32)."""
    v = np.asarray(values, dtype=np.float64) * float(Q16_ONE)
    return np.clip(np.rint(v), -(1 << 31), (1 << 31) - 1).astype(np.int32)


def quantize_fixed_by_scale_q16(values_q16, scale_q16, nonnegative_only: bool = False) -> np.ndarray:
    """Q16.16 values divided by a Q16.16 scale, rounded half to even on the
    integer remainder, clamped to [-127, 127] (or [0, 127])
    (quantize_fixed_tile_by_scale_q16, model/export_fpga_vectors.py:900-927)."""
    den = int(scale_q16) if int(scale_q16) != 0 else 1
    v = np.asarray(values_q16, dtype=np.int64)
    mag = np.abs(v)
    q, r = mag // den, mag % den
    up = (2 * r > den) | ((2 * r == den) & ((q & 1) == 1))
    s = np.where(v < 0, -(q + up), q + up)
    lo = 0 if nonnegative_only else -127
    return np.clip(s, lo, 127).astype(np.int8)


def rmsnorm_contract(x_q, in_scale_q16, gamma_q16, eps: float, out_scale_q16):
    """RMSNorm wrapper (build_rmsnorm_case, model/export_fpga_vectors.py:1705-1728,
    rtl/nonlinear/rmsnorm_wrapper.sv): INT8 x times the Q16.16 input scale,
    the float32 RMSNorm of model/tinyllama.py:45-50 on the dequantized core
    values, Q16.16 result, INT8 output by the Q16.16 output scale. Returns
    (y_q16 int32, y_q int8, y_fp float32)."""
    from . import golden as G
    x_core = np.asarray(x_q, dtype=np.int32) * np.int32(in_scale_q16)
    y_fp = G.rms_norm(float_from_q16_16(x_core), float_from_q16_16(gamma_q16), eps)
    y_q16 = q16_16_signed_array(y_fp)
    return y_q16, quantize_fixed_by_scale_q16(y_q16, out_scale_q16), y_fp


def silu_contract(x_q, in_scale_q16, out_scale_q16):
    """SiLU wrapper (build_silu_case, model/export_fpga_vectors.py:1896-1910,
    rtl/nonlinear/silu_wrapper.sv). Returns (y_q16, y_q, y_fp)."""
    from . import golden as G
    x_core = np.asarray(x_q, dtype=np.int32) * np.int32(in_scale_q16)
    y_fp = G.silu(float_from_q16_16(x_core))
    y_q16 = q16_16_signed_array(y_fp)
    return y_q16, quantize_fixed_by_scale_q16(y_q16, out_scale_q16), y_fp


def softmax_contract(scores_i32, score_scale_q16):
    """Softmax wrapper (build_softmax_case, model/export_fpga_vectors.py:1808-1829,
    rtl/nonlinear/softmax_wrapper.sv:23): INT32 scores times the Q16.16 score
    scale with 32-bit saturation (mul_int32_by_scale_q16, :894-896), float32
    max-shifted softmax of each row (model/tinyllama.py:100-103), Q16.16
    probabilities, INT8 probabilities p * 127 >> 16 rounded half to even and
    clamped to [0, 127] (quantize_probability_q16_tile, :874-888), i.e. the
    1/127 probability scale. Returns (prob_q16, prob_q, prob_fp)."""
    from . import golden as G
    core = np.clip(np.asarray(scores_i32, np.int64) * np.int64(score_scale_q16), -(1 << 31), (1 << 31) - 1)
    fp = float_from_q16_16(core)
    prob = np.stack([G.softmax(r) for r in fp]) if fp.ndim == 2 else G.softmax(fp)
    prob_q16 = q16_16_signed_array(prob)
    p = prob_q16.astype(np.int64) * 127
    r = _round_shift16_half_even(np.abs(p))
    prob_q = np.clip(np.where(p < 0, -r, r), 0, 127).astype(np.int8)
    return prob_q16, prob_q, prob.astype(np.float32)


def residual_add_i32(residual_q16, update_q16) -> np.ndarray:
    """Unsaturated INT32 residual add, wrapping modulo 2**32
    (rtl/compute/residual_add.sv:92-96; build_residual_add_case,
    model/export_fpga_vectors.py:1522-1540)."""
    return (np.asarray(residual_q16, np.int64) + np.asarray(update_q16, np.int64)).astype(np.int32)
