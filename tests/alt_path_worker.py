"""Child process of test_gpu_alt_paths.py: runs one engine configuration
(selected by the TL_DISABLE_* / TL_DECODE_GROUPS variables its parent sets) against the oracle
and exits 0 when every check holds, on a scaled 2-layer model and on one
full-width TinyLlama layer:
* a 300-token prefill layer by layer (tl_decoder_layer), every op checked
  against the oracle on the engine's own inputs (tests/layer_checks.py), and
  the production prefill's hidden state equal to that chain's bit for bit;
* prefill logits, batch-1 generation (the persistent decode kernel, or the
  per-kernel GEMV path with TL_DISABLE_DECODE1=1) and a 48-row batched
  generation (tcgen05 decode, two concurrent row groups of 24 rows unless
  TL_DECODE_GROUPS=1) against the oracle within the sensitivity
  bound of helpers.oracle_run; layer-0 K/V bytes exact.
"""

import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from conftest import load_package  # noqa: E402
from helpers import oracle_run, rel_err, small_model, to_engine_model, tokens_match_modulo_ties  # noqa: E402
from layer_checks import check_kv, check_layer_ops, check_layer_prefix  # noqa: E402
from oracle import golden as G  # noqa: E402
from oracle import weights as W  # noqa: E402
from oracle.kv_golden import KVGolden  # noqa: E402


def run(pkg, qm, tag):
    rng = np.random.default_rng(3)
    eng = pkg.Engine(qm.cfg, max_batch=48, max_prefill_tokens=48 * 16 + 300)
    eng.load(to_engine_model(pkg, qm))
    prompt = [int(t) for t in rng.integers(0, qm.cfg["vocab_size"], 300)]
    ora = KVGolden(qm, kv="int8", matmul=G.ExactMatmul())
    x = qm.embed[np.asarray(prompt)].astype(np.float32)
    for li in range(len(qm.layers)):
        out_e, cap = eng.decoder_layer(li, x, capture=True)
        _, cap_o = ora.layer_capture(li, x)
        check_layer_prefix(cap, cap_o, f"{tag} layer {li}")
        check_kv(eng, ora, li, 300, tag=tag)
        check_layer_ops(cap, x, out_e, qm.layers[li], qm.cfg, cap_o["attended"], per_row=False,
                        tag=f"{tag} layer {li}")
        x = out_e
    hidden = eng.forward_logits(prompt, hidden=True)
    assert np.array_equal(hidden, G.rms_norm(x, qm.final_norm, qm.cfg["rms_norm_eps"])), (tag, "chain vs production")
    ref, ref_logits, bounds, ora = oracle_run(qm, prompt, 6)
    lg = eng.prefill_logits(prompt)
    assert rel_err(lg, ref_logits[0]) <= bounds[0], (tag, "prefill", rel_err(lg, ref_logits[0]), bounds[0])
    k, v, _, _ = eng.read_kv(0, 300)
    assert np.array_equal(k, ora.k_cache[0, :, :300]) and np.array_equal(v, ora.v_cache[0, :, :300]), tag
    toks, st = eng.generate(prompt, 6)
    assert st["generated_count"] == 6 and tokens_match_modulo_ties(toks, ref, ref_logits, bounds), (tag, toks, ref)
    prompts = rng.integers(0, qm.cfg["vocab_size"], (48, 16)).astype(np.uint32)
    outs, sts = eng.generate_batch(prompts, 4)
    assert pkg.shim.load_library().tl_device_error() == 0, tag
    for i in (0, 23, 24, 47):  # first and last row of each row group
        r, rl, b, _ = oracle_run(qm, [int(t) for t in prompts[i]], 4)
        assert tokens_match_modulo_ties(outs[i], r, rl, b), (tag, i, outs[i], r)
    eng.close()


def main():
    pkg = load_package()
    run(pkg, small_model(7, 2), "small")
    dims = W.small_dims(vocab=2048, hidden=2048, ffn=5632, heads=32, kv_heads=4)
    run(pkg, W.random_qmodel(5, 1, dims), "tinyllama-width")
    switches = sorted(k for k in os.environ if k.startswith(("TL_DISABLE_", "TL_DECODE_GROUPS")))
    print("alt path ok:", switches or ["defaults"])


if __name__ == "__main__":
    main()
