"""KV-cached restatement of the golden model: the B200 engine's semantics.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference golden model has no KV cache: ``forward_mixed`` recomputes the
whole prefix at every step and quantizes each activation per tensor across all
rows (model/tinyllama_gemm_int8.py:437-467, 36-42). The hardware spec it models
does keep an INT8 KV cache (docs/design_decisions.txt A7, A10). This module
composes the golden's own blocks (``oracle.golden``) into that cached form:

* Prefill of S prompt tokens is the golden forward on those S rows, unchanged:
  every activation quantized per tensor over the S rows, causal attention, and
  the LM-head input quantized over all S rows before the last row's logits are
  taken. With ``kv="fp32"`` its logits equal ``forward_mixed`` bit for bit.
* With ``kv="int8"`` (the engine's production mode) post-RoPE K and
  post-projection V are stored as symmetric INT8 with one scale per
  (layer, KV head) and tensor: the scale is calibrated on the prompt (the
  :func:`oracle.golden.quantize_int8` rule over that head's [S, head_dim]
  block) and frozen; decode rows reuse it, clamping to +-127. Attention, in
  prefill and decode, always reads the dequantized cache
  ``float32(k_q) * float32(s_K)``.
* A decode step processes one new row: its activations are quantized per
  tensor over that single row, which is what a one-row tensor gives.

Stop rules follow rtl/control/stop_condition_unit.sv:19-37 (host abort > EOS >
``count + 1 >= max_new_tokens`` with 0 meaning no limit) and
rtl/control/prefill_decode_controller.sv:83-198 (an empty prompt is a bad
descriptor; ``max_new_tokens == 0`` in prefill mode runs the prefill only).
"""

from __future__ import annotations

import numpy as np

from . import golden as G

STOP_NONE, STOP_EOS, STOP_MAX_TOKENS, STOP_HOST_ABORT, STOP_INTERNAL_ERR = 0, 1, 2, 3, 4
ERR_NONE, ERR_BAD_DESCRIPTOR, ERR_UNSUPPORTED_MODE = 0, 1, 6
ERR_OUT_OF_RANGE = 17
MODE_PREFILL, MODE_DECODE = 0, 1


class KVGolden:
    """One sequence's engine state: position, INT8 (or float32) KV cache."""

    def __init__(self, model, kv: str = "int8", matmul=G.int8_matmul, attention: str = "f64",
                 noise_seed: int = 0):
        """``attention="f32"`` swaps the reference's float64 attention for
        :func:`oracle.golden.attention_core_f32`, ``attention="noisy"`` for
        :func:`oracle.golden.attention_core_noisy` (seeded by ``noise_seed``);
        both exist only to measure the pipeline's sensitivity."""
        if kv not in ("int8", "fp32"):
            raise ValueError("kv must be 'int8' or 'fp32'")
        if attention not in ("f64", "f32", "noisy"):
            raise ValueError("attention must be 'f64', 'f32' or 'noisy'")
        self.m = model
        self.cfg = model.cfg
        self.kv = kv
        self.matmul = matmul
        self.attention = {"f64": G.attention_core, "f32": G.attention_core_f32}.get(attention)
        if attention == "noisy":
            self.attention = G.attention_core_noisy(noise_seed)
        c = self.cfg
        self.cos, self.sin = G.build_rope_cache(c["max_position_embeddings"], c["head_dim"],
                                                c["rope_theta"])
        self.reset()

    # ------------------------------------------------------------------ state
    def reset(self):
        c = self.cfg
        L, hkv, P, hd = (len(self.m.layers), c["num_key_value_heads"],
                         c["max_position_embeddings"], c["head_dim"])
        dt = np.int8 if self.kv == "int8" else np.float32
        self.k_cache = np.zeros((L, hkv, P, hd), dtype=dt)
        self.v_cache = np.zeros((L, hkv, P, hd), dtype=dt)
        self.k_scale = np.ones((L, hkv), dtype=np.float64)
        self.v_scale = np.ones((L, hkv), dtype=np.float64)
        self.pos = 0
        self.pending = None   # emitted token not yet fed through the layers
        self.trace = []  # optional per-layer capture for debugging

    # -------------------------------------------------------------- KV cache
    def _store_prompt_kv(self, li: int, kh: np.ndarray, vh: np.ndarray):
        s = kh.shape[1]
        for h in range(kh.shape[0]):
            if self.kv == "int8":
                kq, ks = G.quantize_int8(kh[h])
                vq, vs = G.quantize_int8(vh[h])
                self.k_cache[li, h, :s] = kq
                self.v_cache[li, h, :s] = vq
                self.k_scale[li, h] = ks
                self.v_scale[li, h] = vs
            else:
                self.k_cache[li, h, :s] = kh[h]
                self.v_cache[li, h, :s] = vh[h]

    def _store_decode_kv(self, li: int, kh: np.ndarray, vh: np.ndarray, p: int):
        for h in range(kh.shape[0]):
            if self.kv == "int8":
                self.k_cache[li, h, p] = G.quantize_with_scale(kh[h, 0], self.k_scale[li, h])
                self.v_cache[li, h, p] = G.quantize_with_scale(vh[h, 0], self.v_scale[li, h])
            else:
                self.k_cache[li, h, p] = kh[h, 0]
                self.v_cache[li, h, p] = vh[h, 0]

    def _read_kv(self, li: int, n: int):
        if self.kv == "int8":
            ks = self.k_scale[li].astype(np.float32)[:, None, None]
            vs = self.v_scale[li].astype(np.float32)[:, None, None]
            return (self.k_cache[li, :, :n].astype(np.float32) * ks,
                    self.v_cache[li, :, :n].astype(np.float32) * vs)
        return self.k_cache[li, :, :n], self.v_cache[li, :, :n]

    def dequantized_kv(self, li: int, n: int):
        return self._read_kv(li, n)

    # ---------------------------------------------------------------- forward
    def _layer(self, li: int, x: np.ndarray, p0: int, prefill: bool) -> np.ndarray:
        c = self.cfg
        lay = self.m.layers[li]
        s = x.shape[0]
        eps = c["rms_norm_eps"]
        mm = self.matmul
        h = G.rms_norm(x, lay.input_norm, eps)
        q, _, _, _ = G.linear_q(h, lay.q.w_q, lay.q.scale, mm)
        k, _, _, _ = G.linear_q(h, lay.k.w_q, lay.k.scale, mm)
        v, _, _, _ = G.linear_q(h, lay.v.w_q, lay.v.scale, mm)
        qh = G.split_heads(q, c["num_attention_heads"], c["head_dim"])
        kh = G.split_heads(k, c["num_key_value_heads"], c["head_dim"])
        vh = G.split_heads(v, c["num_key_value_heads"], c["head_dim"])
        cos, sin = self.cos[p0:p0 + s], self.sin[p0:p0 + s]
        qh = G.rope(qh, cos, sin)
        kh = G.rope(kh, cos, sin)
        if prefill:
            self._store_prompt_kv(li, kh, vh)
        else:
            self._store_decode_kv(li, kh, vh, p0)
        kd, vd = self._read_kv(li, p0 + s)
        att = self.attention(qh, kd, vd, c["num_key_value_groups"], c["attn_scale"], prefill)
        o, _, _, _ = G.linear_q(att, lay.o.w_q, lay.o.scale, mm)
        x1 = x + o
        h2 = G.rms_norm(x1, lay.post_norm, eps)
        g, _, _, _ = G.linear_q(h2, lay.gate.w_q, lay.gate.scale, mm)
        u, _, _, _ = G.linear_q(h2, lay.up.w_q, lay.up.scale, mm)
        hid = G.silu(g) * u
        d, _, _, _ = G.linear_q(hid, lay.down.w_q, lay.down.scale, mm)
        return (x1 + d).astype(np.float32)

    def layer_capture(self, li: int, x: np.ndarray, p0: int = 0, prefill: bool = True) -> tuple[np.ndarray, dict]:
        """Layer ``li`` on ``x`` recording the tensors the engine's
        ``tl_decoder_layer`` / ``tl_decode_layer`` captures name: each
        projection's INT8 input and its absmax, INT32 accumulators, the float
        projections, the attention output and the block outputs. With
        ``prefill`` ``x`` [S, hidden] is a prompt at positions 0..S-1 (K/V of
        this layer calibrated and cached); otherwise ``x`` [1, hidden] is the
        token at position ``p0`` (K/V quantized with the frozen scales and
        appended). Follows :meth:`_layer` (and through it
        model/tinyllama_gemm_int8.py:136-281)."""
        c = self.cfg
        lay = self.m.layers[li]
        s = x.shape[0]
        eps = c["rms_norm_eps"]
        mm = self.matmul
        cap = {}
        h = G.rms_norm(x, lay.input_norm, eps)
        xq, sx = G.quantize_int8(h)
        cap.update(attn_input=h, qkv_input_q=xq, qkv_input_absmax=np.float32(np.max(np.abs(h))))
        outs = {}
        for name in ("q", "k", "v"):
            ln = getattr(lay, name)
            acc = mm(xq, ln.w_q)
            outs[name] = G.dequantize_int32(acc, sx, ln.scale)
            cap[f"{name}_acc"] = acc
            cap[f"{name}_proj"] = outs[name]
        qh = G.split_heads(outs["q"], c["num_attention_heads"], c["head_dim"])
        kh = G.split_heads(outs["k"], c["num_key_value_heads"], c["head_dim"])
        vh = G.split_heads(outs["v"], c["num_key_value_heads"], c["head_dim"])
        qh = G.rope(qh, self.cos[p0:p0 + s], self.sin[p0:p0 + s])
        kh = G.rope(kh, self.cos[p0:p0 + s], self.sin[p0:p0 + s])
        if prefill:
            self._store_prompt_kv(li, kh, vh)
        else:
            self._store_decode_kv(li, kh, vh, p0)
        cap["q_rot"] = qh
        kd, vd = self._read_kv(li, p0 + s)
        att = self.attention(qh, kd, vd, c["num_key_value_groups"], c["attn_scale"], prefill)
        aq, sa = G.quantize_int8(att)
        acc = mm(aq, lay.o.w_q)
        o = G.dequantize_int32(acc, sa, lay.o.scale)
        cap.update(attended=att.astype(np.float32), o_input_q=aq, o_input_absmax=np.float32(np.max(np.abs(att))),
                   o_acc=acc, o_proj=o)
        x1 = x + o
        h2 = G.rms_norm(x1, lay.post_norm, eps)
        hq, sh = G.quantize_int8(h2)
        cap.update(x_after_attn=x1, ffn_input=h2, gate_up_input_q=hq,
                   gate_up_input_absmax=np.float32(np.max(np.abs(h2))))
        for name in ("gate", "up"):
            ln = getattr(lay, name)
            acc = mm(hq, ln.w_q)
            outs[name] = G.dequantize_int32(acc, sh, ln.scale)
            cap[f"{name}_acc"] = acc
            cap[f"{name}_proj"] = outs[name]
        hid = G.silu(outs["gate"]) * outs["up"]
        dq, sd = G.quantize_int8(hid)
        acc = mm(dq, lay.down.w_q)
        d = G.dequantize_int32(acc, sd, lay.down.scale)
        cap.update(hidden=hid, down_input_q=dq, down_input_absmax=np.float32(np.max(np.abs(hid))),
                   down_acc=acc, down_proj=d)
        return (x1 + d).astype(np.float32), cap

    def _head(self, x: np.ndarray) -> np.ndarray:
        """Final RMSNorm over all rows, per-tensor quantization over all rows,
        logits of the last row only (model/tinyllama_gemm_int8.py:463-467, 671)."""
        hn = G.rms_norm(x, self.m.final_norm, self.cfg["rms_norm_eps"])
        xq, sx = G.quantize_int8(hn)
        acc = self.matmul(xq[-1:], self.m.lm_head.w_q)
        return G.dequantize_int32(acc, sx, self.m.lm_head.scale)[0]

    def prefill(self, ids) -> np.ndarray:
        ids = list(ids)
        if not ids:
            raise ValueError("empty prompt")
        if len(ids) > self.cfg["max_position_embeddings"]:
            raise ValueError("prompt longer than max_position_embeddings")
        self.reset()
        x = self.m.embed[np.asarray(ids)].astype(np.float32)
        for li in range(len(self.m.layers)):
            x = self._layer(li, x, 0, True)
        self.pos = len(ids)
        self.pending = None
        return self._head(x)

    def decode(self, token: int) -> np.ndarray:
        if self.pos >= self.cfg["max_position_embeddings"]:
            raise IndexError("KV cache full")
        x = self.m.embed[np.asarray([token])].astype(np.float32)
        for li in range(len(self.m.layers)):
            x = self._layer(li, x, self.pos, False)
        self.pos += 1
        self.pending = None
        return self._head(x)

    # --------------------------------------------------------------- runtime
    def generate(self, prompt, max_new_tokens: int, eos_id: int, mode: int = MODE_PREFILL,
                 abort_after=None, out_cap: int | None = None):
        """Greedy generation with the RTL stop contract.

        Returns (tokens, stop_reason, error_code). ``abort_after=n`` raises the
        host abort once n tokens have been emitted (it is checked before each
        further step, as the controller samples ABORT in every state)."""
        prompt = list(prompt)
        cap = out_cap if out_cap is not None else (1 << 30)
        if mode not in (MODE_PREFILL, MODE_DECODE):
            return [], STOP_NONE, ERR_UNSUPPORTED_MODE
        out: list[int] = []
        if mode == MODE_PREFILL:
            if not prompt:
                return [], STOP_NONE, ERR_BAD_DESCRIPTOR
            if len(prompt) > self.cfg["max_position_embeddings"]:
                return [], STOP_INTERNAL_ERR, ERR_OUT_OF_RANGE
            logits = self.prefill(prompt)
            if max_new_tokens == 0:
                return [], STOP_NONE, ERR_NONE
        else:
            if self.pending is None and not prompt:
                return [], STOP_NONE, ERR_BAD_DESCRIPTOR
            feed = prompt if prompt else [self.pending]
            logits = None
            for t in feed:
                if self.pos >= self.cfg["max_position_embeddings"]:
                    return [], STOP_INTERNAL_ERR, ERR_OUT_OF_RANGE
                logits = self.decode(t)
        limit = max_new_tokens if max_new_tokens != 0 else cap
        limit = min(limit, cap)
        while True:
            if abort_after is not None and len(out) >= abort_after:
                return out, STOP_HOST_ABORT, ERR_NONE
            tok = G.argmax_first(logits)
            out.append(tok)
            self.pending = tok
            if tok == eos_id:
                return out, STOP_EOS, ERR_NONE
            if len(out) >= limit:
                return out, STOP_MAX_TOKENS, ERR_NONE
            if self.pos >= self.cfg["max_position_embeddings"]:
                return out, STOP_INTERNAL_ERR, ERR_OUT_OF_RANGE
            logits = self.decode(tok)
