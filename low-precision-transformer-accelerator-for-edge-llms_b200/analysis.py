"""Accuracy report of the INT8 engine against the float32 model: the
reference's ``run_analysis`` / ``dump_debug`` tooling
(model/tinyllama_gemm_int8.py:470-626, :302-327) over the B200 engine.

Per layer, as the reference does:
* isolated: the float32 layer and the engine's INT8 layer on the same float32
  input (the float32 model's layer input);
* cumulative: the engine's INT8 layer on the INT8 path's own previous
  output;
MAE and max |diff| of both against the float32 layer output
(``diff_stats``, :48-56), a per-projection breakdown for the dumped layer,
final-logit MAE / RMSE / max |diff|, both next tokens and both top-k lists.
The INT8 side is the engine (``Engine.decoder_layer``, per-tensor weights as
the reference bridge quantizes them, its INT8 KV cache in attention); its
last-row LM head is ``quantized_linear`` on that one row, as the reference's
report computes it (:573-580). The float32 side is the reference's
``reference_decoder_layer`` (:228-253) restated in PyTorch float32 on the
GPU (TF32 off; scores, softmax and weighted sum in float64 as the
reference's float64 ``attn_scale`` makes them): the baseline of the
comparison, not an engine path.

``dump_dir`` writes ``debug_arrays.npz`` (``token_ids``, then every array of
the dumped layer's float32 and INT8 debug dictionaries flattened with the
reference's ``flatten_named_arrays`` key rule under ``reference_`` /
``mixed_``, plus ``mixed_lm_head_*``) and ``summary.txt``.
"""

from __future__ import annotations

import os
from typing import Any, Callable

import numpy as np

from . import shim


def diff_stats(reference, candidate) -> dict:
    """MAE, RMSE and max |diff| in float32 (model/tinyllama_gemm_int8.py:48-56)."""
    diff = np.asarray(candidate, dtype=np.float32) - np.asarray(reference, dtype=np.float32)
    ad = np.abs(diff)
    return {"mae": float(ad.mean()), "rmse": float(np.sqrt(np.mean(diff * diff))), "max_abs": float(ad.max())}


def flatten_named_arrays(prefix: str, obj: Any) -> dict:
    """Nested debug dict -> flat ``prefix_key_subkey`` arrays
    (model/tinyllama_gemm_int8.py:302-310)."""
    flat: dict = {}
    if isinstance(obj, dict):
        for k, v in obj.items():
            flat.update(flatten_named_arrays(f"{prefix}_{k}" if prefix else k, v))
    elif isinstance(obj, np.ndarray):
        flat[prefix] = obj
    return flat


def dump_debug(dump_dir: str, token_ids, reference_debug: dict, mixed_debug: dict, summary_lines) -> None:
    """debug_arrays.npz + summary.txt (model/tinyllama_gemm_int8.py:313-327)."""
    os.makedirs(dump_dir, exist_ok=True)
    arrays = {"token_ids": np.asarray(token_ids, dtype=np.int32)}
    arrays.update(flatten_named_arrays("reference", reference_debug))
    arrays.update(flatten_named_arrays("mixed", mixed_debug))
    np.savez(os.path.join(dump_dir, "debug_arrays.npz"), **arrays)
    with open(os.path.join(dump_dir, "summary.txt"), "w", encoding="utf-8") as fh:
        fh.write("\n".join(summary_lines) + "\n")


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device visible: the analysis runs on the GPU")
    return torch


def reference_decoder_layer(x, layer: dict, cfg: dict, cos, sin, capture_arrays: bool = False):
    """Float32 decoder layer (model/tinyllama_gemm_int8.py:91-133, 185-253) in
    PyTorch on the GPU. Returns (out float32 [S, hidden], debug dict with the
    reference's keys)."""
    torch = _torch()
    dev = torch.device("cuda")

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32))).to(dev)

    def rms(v, w):
        return v * (1.0 / torch.sqrt(torch.mean(v * v, dim=-1, keepdim=True) + cfg["rms_norm_eps"])) * t(w)

    def lin(v, name):
        out = v @ t(layer[f"{name}_w"])
        b = layer.get(f"{name}_b")
        return out if b is None else out + t(b)

    def rope(h, s):
        c, sn = t(cos[:s])[None], t(sin[:s])[None]
        half = h.shape[-1] // 2
        rot = torch.cat([-h[..., half:], h[..., :half]], dim=-1)
        return h * c + rot * sn

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xs = t(x)
        s = xs.shape[0]
        H, Hkv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
        attn_in = rms(xs, layer["input_norm_w"])
        q, k, v = lin(attn_in, "q"), lin(attn_in, "k"), lin(attn_in, "v")
        qh = rope(q.reshape(s, H, hd).transpose(0, 1), s)
        kh = rope(k.reshape(s, Hkv, hd).transpose(0, 1), s)
        vh = v.reshape(s, Hkv, hd).transpose(0, 1)
        g = H // Hkv
        kr = kh.repeat_interleave(g, dim=0)
        vr = vh.repeat_interleave(g, dim=0)
        scores = (qh @ kr.transpose(1, 2)).double() * float(cfg["attn_scale"])
        mask = torch.ones(s, s, dtype=torch.bool, device=dev).tril()
        scores = scores.masked_fill(~mask, -1e9)
        probs = torch.softmax(scores, dim=-1)
        attended = (probs @ vr.double()).transpose(0, 1).reshape(s, H * hd).float()
        attn_out = lin(attended, "o")
        x1 = xs + attn_out
        ffn_in = rms(x1, layer["post_norm_w"])
        gate, up = lin(ffn_in, "gate"), lin(ffn_in, "up")
        hid = gate / (1.0 + torch.exp(-torch.clamp(gate, -60.0, 60.0))) * up
        ffn_out = lin(hid, "down")
        out = x1 + ffn_out
        n = lambda a: a.detach().cpu().numpy()
        attn = {"q_proj_fp": n(q), "k_proj_fp": n(k), "v_proj_fp": n(v)}
        ffn = {"gate_proj_fp": n(gate), "up_proj_fp": n(up), "hidden_fp": n(hid)}
        if capture_arrays:
            attn.update({"scores_fp": n(scores), "weights_fp": n(probs), "attended_fp": n(attended),
                         "out_fp": n(attn_out)})
            ffn["out_fp"] = n(ffn_out)
        debug = {"attn_input_fp": n(attn_in), "x_after_attn_fp": n(x1), "ffn_input_fp": n(ffn_in),
                 "attn": attn, "ffn": ffn}
        if capture_arrays:
            debug["layer_out_fp"] = n(out)
        return n(out).astype(np.float32), debug
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def top_tokens(logits, k: int, decode: Callable[[int], str] | None = None) -> list:
    """k largest logits, highest first: (id, value, text) (:289-294)."""
    idx = np.argsort(logits)[-k:][::-1]
    return [(int(i), float(logits[i]), decode(int(i)) if decode else "") for i in idx]


def run_analysis(token_ids, weights, layer_count: int = 1, dump_layer: int | None = None,
                 dump_dir: str | None = None, top_k: int = 10, quantize_lm_head: bool = True,
                 decode: Callable[[int], str] | None = None, print_fn: Callable[[str], None] | None = print) -> dict:
    """The reference's ``run_analysis`` (model/tinyllama_gemm_int8.py:470-626)
    with the INT8 side on the engine. ``weights`` is a ``TinyLlamaWeights``-
    like object (``cfg``, ``layer(i)``, ``embed``/``_array``,
    ``final_norm_w()``, ``lm_head_w()``); ``decode`` maps a token id to its
    text (the tokenizer's, when one is available). Prints the reference's
    lines (through ``print_fn``) and returns them with the numbers."""
    cfg = dict(weights.cfg)
    if layer_count < 1 or layer_count > cfg["num_hidden_layers"]:
        raise ValueError(f"--layers must be between 1 and {cfg['num_hidden_layers']}")
    if dump_layer is not None and (dump_layer < 0 or dump_layer >= layer_count):
        raise ValueError("--dump-layer must be within the executed layer range")
    token_ids = [int(t) for t in token_ids]
    if not token_ids:
        raise ValueError("Input token sequence is empty")
    say = print_fn or (lambda _line: None)
    say(f"Token ids: {token_ids}")
    say("")
    emb = weights._array("embed_w") if hasattr(weights, "_array") else weights.embed_w
    x_ref = np.asarray(emb, np.float32)[np.asarray(token_ids)].astype(np.float32)
    x_mix = x_ref.copy()
    cos, sin = shim.rope_tables(cfg["max_position_embeddings"], cfg["head_dim"], cfg["rope_theta"])
    eng = shim._cached_engine(("model", id(weights), layer_count), weights,
                              lambda: shim.from_tinyllama_weights(weights, layer_count),
                              cfg, cfg["max_position_embeddings"])
    summary = [f"Token ids: {token_ids}", f"Layers analyzed: {layer_count}", "Layer stats:"]
    layers_out, dump_ref, dump_mix = [], None, None
    fields_all = [n for n, _, _ in shim.CAPTURE_FIELDS]
    fields = [n for n, _, k in shim.CAPTURE_FIELDS if k != "HSS"]
    for li in range(layer_count):
        layer = weights.layer(li)
        capture = dump_layer == li
        ref_out, ref_dbg = reference_decoder_layer(x_ref, layer, cfg, cos, sin, capture_arrays=capture)
        iso_out, iso_cap = eng.decoder_layer(li, x_ref, capture=fields_all if capture else fields)
        cum_out, _ = eng.decoder_layer(li, x_mix)
        iso = diff_stats(ref_out, iso_out)
        cum = diff_stats(ref_out, cum_out)
        line = (f"Layer {li}: isolated MAE={iso['mae']:.6f}, isolated max={iso['max_abs']:.6f}, "
                f"cumulative MAE={cum['mae']:.6f}, cumulative max={cum['max_abs']:.6f}")
        say(line)
        summary.append(line)
        layers_out.append({"layer": li, "isolated": iso, "cumulative": cum})
        if capture:
            quant = {p: shim.quantize_weight(layer[f"{p}_w"], "tensor") for p in shim._NPZ_PROJ}
            wfp = {p: np.asarray(layer[f"{p}_w"], np.float32) for p in shim._NPZ_PROJ}
            iso_dbg = shim.layer_debug(iso_cap, True, wfp, quant)
            iso_dbg["layer_out_fp"] = iso_out
            dump_ref, dump_mix = ref_dbg, iso_dbg
            pairs = [("  attn q_proj", "attn", "q_proj_fp"), ("  attn k_proj", "attn", "k_proj_fp"),
                     ("  attn v_proj", "attn", "v_proj_fp"), ("  ffn gate_proj", "ffn", "gate_proj_fp"),
                     ("  ffn up_proj", "ffn", "up_proj_fp"), ("  attn o_proj", "attn", "out_fp"),
                     ("  ffn down_proj", "ffn", "out_fp")]
            breakdown = {}
            for name, blk, key in pairs:
                st = diff_stats(ref_dbg[blk][key], iso_dbg[blk][key])
                breakdown[name.strip()] = st
                bl = f"{name}: mae={st['mae']:.6f}, max_abs={st['max_abs']:.6f}"
                say(bl)
                summary.append(bl)
            layers_out[-1]["breakdown"] = breakdown
        x_ref, x_mix = ref_out, cum_out
    torch = _torch()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        lm_w = np.asarray(weights.lm_head_w(), np.float32)
        gamma = np.asarray(weights.final_norm_w(), np.float32)
        g = torch.from_numpy(gamma).cuda()
        xt = torch.from_numpy(np.ascontiguousarray(x_ref)).cuda()
        xn = xt * (1.0 / torch.sqrt(torch.mean(xt * xt, dim=-1, keepdim=True) + cfg["rms_norm_eps"])) * g
        ref_logits = (xn[-1:] @ torch.from_numpy(lm_w).cuda()).cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    x_mix_n = shim.rms_norm(x_mix, weights.final_norm_w(), cfg["rms_norm_eps"])
    lm_dbg: dict = {}
    if quantize_lm_head:
        mix_logits, lm_dbg = shim.quantized_linear(x_mix_n[-1:], lm_w, None, capture_arrays=dump_dir is not None)
    else:
        mix_logits = (x_mix_n[-1:] @ lm_w).astype(np.float32)
    ls = diff_stats(ref_logits, mix_logits)
    ref_tok, mix_tok = int(np.argmax(ref_logits[0])), int(np.argmax(mix_logits[0]))
    txt = (lambda i: decode(i)) if decode else (lambda i: "")
    say("")
    say(f"Final logits: MAE={ls['mae']:.6f}, RMSE={ls['rmse']:.6f}, max_abs={ls['max_abs']:.6f}")
    say(f"Float32 next token: {ref_tok} -> '{txt(ref_tok)}'")
    say(f"INT8 path next token: {mix_tok} -> '{txt(mix_tok)}'")
    top_ref, top_mix = top_tokens(ref_logits[0], top_k, decode), top_tokens(mix_logits[0], top_k, decode)
    for title, rows in ((f"Top {top_k} float32 tokens:", top_ref), (f"Top {top_k} INT8-path tokens:", top_mix)):
        say("")
        say(title)
        for i, v, s in rows:
            say(f"  {i:6d}  {v:12.6f}  '{s}'")
    summary.extend(["", f"Final logits: mae={ls['mae']:.6f}, rmse={ls['rmse']:.6f}, max_abs={ls['max_abs']:.6f}",
                    f"Float32 next token: {ref_tok} -> '{txt(ref_tok)}'",
                    f"INT8 path next token: {mix_tok} -> '{txt(mix_tok)}'"])
    if dump_dir is not None:
        mixed = dict(dump_mix or {})
        if quantize_lm_head and lm_dbg:
            mixed["lm_head"] = lm_dbg
        dump_debug(dump_dir, token_ids, dump_ref or {}, mixed, summary)
        say("")
        say(f"Saved debug dump to {dump_dir}")
    return {"layers": layers_out, "logits": ls, "ref_logits": ref_logits, "mix_logits": mix_logits,
            "ref_token": ref_tok, "mix_token": mix_tok, "top_ref": top_ref, "top_mix": top_mix,
            "summary": summary}
