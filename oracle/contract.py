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
