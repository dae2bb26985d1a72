"""Op-by-op checks of one engine decoder layer (tests only).

``check_layer_ops`` compares every op of a ``tl_decoder_layer`` /
``tl_decode_layer`` capture with the oracle's op applied to the ENGINE's own
input of that op, so a float difference upstream cannot hide or excuse an
error downstream:

* exact: RMSNorm outputs, each INT8 quantization (values and absmax, per
  tensor over the sequence in prefill, per row in decode), every INT32
  accumulator (exact product of the engine's INT8 input and the weight),
  every dequantized projection, both residual adds;
* attention output within 1e-5 of the float64 oracle on the same q and
  cache, SiLU*up within 1e-6 (the device's expf vs NumPy's exp).

``check_layer_prefix`` compares the part of the layer that is exact end to
end with the oracle's own run of the layer on the same input: the
projections' INT8 input, their accumulators, and the INT8 K/V bytes.
"""

from __future__ import annotations

import numpy as np

from oracle import golden as G

ATTN_RTOL = 1e-5
SILU_RTOL = 1e-6


def _groups(a, per_row: bool):
    a = np.asarray(a)
    return [a[i:i + 1] for i in range(a.shape[0])] if per_row else [a]


def _quant_check(name, fp, q, absmax, per_row):
    """q / absmax must be the engine quantizer's output for its own float
    input fp (model/tinyllama_gemm_int8.py:36-42 over the group)."""
    for gi, (xf, xq) in enumerate(zip(_groups(fp, per_row), _groups(q, per_row))):
        want_q, _ = G.quantize_int8(xf)
        np.testing.assert_array_equal(xq, want_q, err_msg=f"{name} INT8 values, group {gi}")
        assert absmax[gi] == np.float32(np.max(np.abs(xf))), (name, gi, absmax[gi], np.max(np.abs(xf)))


def _scales(absmax, rows, per_row):
    s = [1.0 if float(a) == 0.0 else float(a) / 127.0 for a in absmax]
    return s if per_row else s * rows


def _linear_check(name, q, absmax, acc, proj, lin, per_row):
    want = G.int8_matmul(q, lin.w_q)
    np.testing.assert_array_equal(acc, want, err_msg=f"{name} INT32 accumulators")
    sx = _scales(absmax, q.shape[0], per_row)
    for r in range(q.shape[0]):
        np.testing.assert_array_equal(proj[r], G.dequantize_int32(want[r], sx[r], lin.scale),
                                      err_msg=f"{name} dequantized row {r}")


def check_layer_ops(cap, x, out, lay, cfg, attended_ref, per_row: bool, tag=""):
    """Every op of one captured layer against the oracle op applied to the
    engine's own inputs. ``attended_ref`` is the float64 oracle attention on
    the same q rows and the same K/V cache."""
    eps = cfg["rms_norm_eps"]
    np.testing.assert_array_equal(cap["attn_input"], G.rms_norm(x, lay.input_norm, eps), err_msg=f"{tag} input norm")
    _quant_check(f"{tag} qkv input", cap["attn_input"], cap["qkv_input_q"], cap["qkv_input_absmax"], per_row)
    for p in ("q", "k", "v"):
        _linear_check(f"{tag} {p}_proj", cap["qkv_input_q"], cap["qkv_input_absmax"], cap[f"{p}_acc"],
                      cap[f"{p}_proj"], getattr(lay, p), per_row)
    att = cap["attended"]
    err = np.max(np.abs(att - attended_ref)) / max(np.max(np.abs(attended_ref)), 1e-30)
    assert err <= ATTN_RTOL, (tag, "attention", err)
    _quant_check(f"{tag} o input", att, cap["o_input_q"], cap["o_input_absmax"], per_row)
    _linear_check(f"{tag} o_proj", cap["o_input_q"], cap["o_input_absmax"], cap["o_acc"], cap["o_proj"], lay.o,
                  per_row)
    np.testing.assert_array_equal(cap["x_after_attn"], x + cap["o_proj"], err_msg=f"{tag} attention residual")
    np.testing.assert_array_equal(cap["ffn_input"], G.rms_norm(cap["x_after_attn"], lay.post_norm, eps),
                                  err_msg=f"{tag} post norm")
    _quant_check(f"{tag} gate/up input", cap["ffn_input"], cap["gate_up_input_q"], cap["gate_up_input_absmax"],
                 per_row)
    for p in ("gate", "up"):
        _linear_check(f"{tag} {p}_proj", cap["gate_up_input_q"], cap["gate_up_input_absmax"], cap[f"{p}_acc"],
                      cap[f"{p}_proj"], getattr(lay, p), per_row)
    hid_ref = G.silu(cap["gate_proj"]) * cap["up_proj"]
    err = np.max(np.abs(cap["hidden"] - hid_ref)) / max(np.max(np.abs(hid_ref)), 1e-30)
    assert err <= SILU_RTOL, (tag, "silu*up", err)
    _quant_check(f"{tag} down input", cap["hidden"], cap["down_input_q"], cap["down_input_absmax"], per_row)
    _linear_check(f"{tag} down_proj", cap["down_input_q"], cap["down_input_absmax"], cap["down_acc"],
                  cap["down_proj"], lay.down, per_row)
    np.testing.assert_array_equal(out, cap["x_after_attn"] + cap["down_proj"], err_msg=f"{tag} ffn residual")


def check_layer_prefix(cap, cap_o, tag="", row=None):
    """The exact prefix against the oracle's own run of the layer on the same
    input (``row`` selects one engine row for a decode capture)."""
    sel = (lambda a: a) if row is None else (lambda a: np.asarray(a)[row:row + 1])
    for k in ("attn_input", "qkv_input_q", "q_acc", "k_acc", "v_acc", "q_proj", "k_proj", "v_proj"):
        np.testing.assert_array_equal(sel(cap[k]), cap_o[k], err_msg=f"{tag} {k}")
    got = np.asarray(cap["qkv_input_absmax"])[0 if row is None else row]
    assert got == cap_o["qkv_input_absmax"], (tag, got, cap_o["qkv_input_absmax"])


def check_kv(eng, ora, li, n, slot=0, tag=""):
    """INT8 K/V bytes and scales of layer li, positions 0..n-1."""
    k, v, ks, vs = eng.read_kv(li, n, slot=slot)
    np.testing.assert_array_equal(k, ora.k_cache[li, :, :n], err_msg=f"{tag} layer {li} K cache")
    np.testing.assert_array_equal(v, ora.v_cache[li, :, :n], err_msg=f"{tag} layer {li} V cache")
    np.testing.assert_array_equal(ks, ora.k_scale[li].astype(np.float32), err_msg=f"{tag} K scales")
    np.testing.assert_array_equal(vs, ora.v_scale[li].astype(np.float32), err_msg=f"{tag} V scales")
