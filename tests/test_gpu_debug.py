"""Step-scoped debug capture (GPU): tl_decode_debug returns the fixed tensor
set of the hardware's debug contract (docs/design_decisions.txt B8) for one
layer of a decode step. Each field is checked against the oracle applied to
the engine's own captured inputs, with the oracle's cache loaded from the
engine's (so both hold the same state): the quantized q/k/v input, the
projections and the updated K/V cache rows exact; score / probability
windows against float64 (1e-5 / 1e-6); the final hidden state exact from the
last layer's output; the top-16 logits and the chosen token exact from the
final hidden state (INT8 LM head)."""

import numpy as np
import pytest

from oracle import golden as G
from oracle.kv_golden import KVGolden

from helpers import rel_err, small_model, to_engine_model

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_decode_debug_capture(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    qm = small_model(23, 2)
    c = qm.cfg
    eng = pkg.Engine(c, max_batch=1, max_prefill_tokens=64)
    eng.load(to_engine_model(pkg, qm))
    prompt = [int(t) for t in np.random.default_rng(24).integers(0, c["vocab_size"], 20)]
    lg = eng.prefill_logits(prompt)
    tok = int(np.argmax(lg))
    ora = KVGolden(qm, kv="int8", matmul=G.ExactMatmul())
    for li in range(2):
        k, v, ks, vs = eng.read_kv(li, 20)
        ora.k_cache[li, :, :20], ora.v_cache[li, :, :20] = k, v
        ora.k_scale[li], ora.v_scale[li] = ks, vs
    # layer 0 of the step at position 20
    r0 = eng.decode_debug(tok, 0, logits=True)
    assert r0["position"] == 20 and eng.position() == 21
    np.testing.assert_array_equal(r0["layer_input"], qm.embed[tok])
    _, cap = ora.layer_capture(0, r0["layer_input"][None], p0=20, prefill=False)
    np.testing.assert_array_equal(r0["qkv_input_q"], cap["qkv_input_q"][0])
    assert r0["input_absmax"][0] == cap["qkv_input_absmax"]
    for f in ("q_proj", "k_proj", "v_proj"):
        np.testing.assert_array_equal(r0[f], cap[f][0])
    np.testing.assert_array_equal(r0["k_row"], ora.k_cache[0, :, 20])
    np.testing.assert_array_equal(r0["v_row"], ora.v_cache[0, :, 20])
    np.testing.assert_array_equal(r0["k_scale"], ora.k_scale[0].astype(np.float32))
    kd, _ = ora.dequantized_kv(0, 21)
    sc = (cap["q_rot"] @ G.repeat_kv(kd, c["num_key_value_groups"]).transpose(0, 2, 1))[:, 0] * c["attn_scale"]
    assert np.max(np.abs(r0["scores"] - sc)) <= 1e-5 * np.max(np.abs(sc))
    assert np.max(np.abs(r0["probs"] - G.softmax(sc))) <= 1e-6
    assert rel_err(r0["attended"], cap["attended"][0]) <= 1e-5
    assert r0["input_absmax"][1] == np.max(np.abs(r0["attended"]))
    assert rel_err(r0["layer_output"], ora._layer(0, r0["layer_input"][None], 20, False)[0]) <= 2e-2
    # last layer of the next step: final hidden, top-16 and token follow exactly from its output
    nxt = r0["chosen_token"]
    assert nxt == G.argmax_first(r0["logits"])
    r1 = eng.decode_debug(nxt, 1)
    assert r1["position"] == 21
    np.testing.assert_array_equal(r1["final_hidden"], G.rms_norm(r1["layer_output"], qm.final_norm, c["rms_norm_eps"]))
    assert r1["input_absmax"][4] == np.max(np.abs(r1["final_hidden"]))
    hq, sh = G.quantize_int8(r1["final_hidden"])
    logits = G.dequantize_int32(G.int8_matmul(hq[None], qm.lm_head.w_q), sh, qm.lm_head.scale)[0]
    order = sorted(range(len(logits)), key=lambda i: (-logits[i], i))[:16]
    np.testing.assert_array_equal(r1["top_ids"], order)
    np.testing.assert_array_equal(r1["top_logits"], logits[order])
    assert r1["chosen_token"] == order[0]
    assert r1["scores"].shape == (c["num_attention_heads"], 22)
    with pytest.raises(pkg.TLError):
        eng.decode_debug(nxt, 2)
    eng.close()
