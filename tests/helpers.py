"""Shared test helpers: oracle models -> engine models, tolerances."""

from __future__ import annotations

import numpy as np

from oracle import golden as G
from oracle import weights as W
from oracle.kv_golden import KVGolden

# Higher-precision blocks: within 1e-3 relative (of the tensor's magnitude).
FP_RTOL = 1e-3


def to_engine_model(pkg, qm):
    """oracle.weights.QModel -> shim.Model (same arrays, no copy of values)."""
    L = pkg.shim.Linear
    layers = [pkg.shim.Layer(L(l.q.w_q, l.q.scale), L(l.k.w_q, l.k.scale), L(l.v.w_q, l.v.scale),
                             L(l.o.w_q, l.o.scale), L(l.gate.w_q, l.gate.scale), L(l.up.w_q, l.up.scale),
                             L(l.down.w_q, l.down.scale), l.input_norm, l.post_norm) for l in qm.layers]
    return pkg.shim.Model(dict(qm.cfg), qm.embed, qm.final_norm, L(qm.lm_head.w_q, qm.lm_head.scale), layers)


def small_model(seed: int = 7, layers: int = 2, granularity: str = "tensor"):
    return W.quantize_archive(W.random_archive(seed, layers, W.small_dims(), gamma_one=False), granularity)


def rel_close(a, b, rtol=FP_RTOL) -> bool:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = max(np.max(np.abs(b)), 1e-30)
    return float(np.max(np.abs(a - b))) <= rtol * scale


def rel_err(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def tokens_match_modulo_ties(eng_tokens, ref_tokens, ref_logits_per_step, rtol=FP_RTOL) -> bool:
    """Greedy ids must agree step by step, except where the reference's top-2
    logits differ by less than rtol (relative; one value, or one per step);
    comparison stops there."""
    for i, (a, b) in enumerate(zip(eng_tokens, ref_tokens)):
        if a == b:
            continue
        r = rtol[i] if np.ndim(rtol) else rtol
        lg = np.asarray(ref_logits_per_step[i], np.float64)
        top2 = np.sort(lg)[-2:]
        return (top2[1] - top2[0]) <= r * max(abs(top2[1]), 1e-30)
    return len(eng_tokens) == len(ref_tokens)


SENS_FACTOR = 3.0


def oracle_run(qm, prompt, n, matmul=None, noise_seed=0):
    """Greedy run of the KV-cached oracle for ``n`` tokens, plus the bound the
    engine's logits are held to at each step.

    The reference's pipeline re-quantizes every activation to INT8, so an
    attention result that differs from its float64 one by ~1e-6 flips some
    INT8 values by 1 LSB, and those flips propagate (by ~1% per flip on a
    small model, to ~8% over 22 layers). The bound at each step is
    max(1e-3, 3 x the distance between the oracle and the same oracle with
    its attention output perturbed at the CUDA kernels' stated accuracy,
    2e-6 of its maximum; G.attention_core_noisy), the perturbed run
    teacher-forced on the same ids. Returns (ids, logits, bounds, oracle)."""
    mm = matmul or G.ExactMatmul()
    o64 = KVGolden(qm, kv="int8", matmul=mm)
    onz = KVGolden(qm, kv="int8", matmul=mm, attention="noisy", noise_seed=noise_seed)
    l64, lnz = [o64.prefill(prompt)], [onz.prefill(prompt)]
    toks = []
    while True:
        toks.append(G.argmax_first(l64[-1]))
        if len(toks) == n:
            break
        l64.append(o64.decode(toks[-1]))
        lnz.append(onz.decode(toks[-1]))
    bounds = [max(FP_RTOL, SENS_FACTOR * rel_err(b, a)) for a, b in zip(l64, lnz)]
    return toks, l64, bounds, o64
