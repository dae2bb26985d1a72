"""Pin the CPU oracle against the reference's own outputs (CPU only).

The fixtures under tests/golden/ were produced by running the reference's
Python golden model and exporter (tests/golden/make_fixtures.py). Every check
here is bit-exact unless it says otherwise.
"""

import numpy as np
import pytest

from oracle import contract as C
from oracle import golden as G
from oracle import weights as W
from oracle.kv_golden import KVGolden


def test_quantize_int8_matches_reference(golden):
    d = golden["quant_cases"]
    keys = sorted({k.split("_")[0] for k in d.files if k.startswith("q")})
    assert len(keys) >= 7
    for key in keys:
        q, s = G.quantize_int8(d[f"{key}_x"])
        np.testing.assert_array_equal(q, d[f"{key}_q"], err_msg=key)
        assert s == float(d[f"{key}_scale"]), key


def test_quantized_linear_matches_reference(golden):
    d = golden["quant_cases"]
    for i in range(4):
        out, dbg = G.quantized_linear(d[f"l{i}_x"], d[f"l{i}_w"])
        np.testing.assert_array_equal(dbg["input_q"], d[f"l{i}_xq"])
        np.testing.assert_array_equal(dbg["weight_q"], d[f"l{i}_wq"])
        np.testing.assert_array_equal(dbg["accum_int32"], d[f"l{i}_acc"])
        np.testing.assert_array_equal(out, d[f"l{i}_out"])
        # pre-quantized per-tensor weights give the identical output
        lq = W.quantize_weight(d[f"l{i}_w"], "tensor")
        out2, _, _, acc2 = G.linear_q(d[f"l{i}_x"], lq.w_q, lq.scale)
        np.testing.assert_array_equal(acc2, d[f"l{i}_acc"])
        np.testing.assert_array_equal(out2, d[f"l{i}_out"])


def test_exact_matmul_equals_int32_path():
    rng = np.random.default_rng(3)
    a = rng.integers(-127, 128, (5, 5632)).astype(np.int8)
    b = rng.integers(-127, 128, (5632, 33)).astype(np.int8)
    np.testing.assert_array_equal(G.int8_matmul(a, b), G.int8_matmul_reference_path(a, b))
    # worst case magnitude: all +-127
    a = np.full((2, 5632), -127, np.int8)
    b = np.full((5632, 3), 127, np.int8)
    np.testing.assert_array_equal(G.int8_matmul(a, b), G.int8_matmul_reference_path(a, b))


def test_pairwise_sum_is_numpy_order():
    rng = np.random.default_rng(11)
    for n in (1, 7, 8, 9, 64, 127, 128, 129, 300, 2048, 5632):
        for _ in range(4):
            v = (rng.standard_normal(n, dtype=np.float32) * rng.uniform(1e-3, 1e3)).astype(np.float32)
            sq = v * v
            assert G.pairwise_sum_f32(sq) == np.sum(sq), n


def test_rmsnorm_rope_silu_match_reference(golden):
    d = golden["small_model"]
    np.testing.assert_array_equal(G.rms_norm(d["rms_x"], d["rms_g"], 1e-5), d["rms_out"])
    np.testing.assert_array_equal(G.silu(d["silu_x"]), d["silu_out"])
    c, s = G.build_rope_cache(64, 64, 10000.0)
    np.testing.assert_array_equal(c, d["rope_cos"])
    np.testing.assert_array_equal(s, d["rope_sin"])


def _small_model(d):
    arc = W.random_archive(int(d["seed"]), int(d["layers"]), W.small_dims(), gamma_one=False)
    return W.quantize_archive(arc, "tensor")


def test_small_model_forward_matches_reference(golden):
    d = golden["small_model"]
    m = _small_model(d)
    cos, sin = G.build_rope_cache(m.cfg["max_position_embeddings"], 64, m.cfg["rope_theta"])
    prompt = [int(t) for t in d["prompt"]]
    np.testing.assert_array_equal(G.forward_mixed(prompt, m, cos, sin), d["prompt_logits"])
    x = m.embed[np.asarray(prompt)]
    np.testing.assert_array_equal(G.decoder_layer_mixed(x, m.layers[0], m.cfg, cos, sin), d["layer0_out"])
    # per-projection INT32 accumulators of layer 0 (the reference's debug capture)
    h = G.rms_norm(x, m.layers[0].input_norm, m.cfg["rms_norm_eps"])
    np.testing.assert_array_equal(h, d["layer0_attn_input"])
    for name, lin in (("q_proj", m.layers[0].q), ("k_proj", m.layers[0].k), ("v_proj", m.layers[0].v)):
        _, xq, _, acc = G.linear_q(h, lin.w_q, lin.scale)
        np.testing.assert_array_equal(xq, d[f"layer0_{name}_xq"])
        np.testing.assert_array_equal(acc, d[f"layer0_{name}_acc"])
    toks = G.generate_recompute(prompt, m, cos, sin, len(d["recompute_tokens"]))
    assert toks == [int(t) for t in d["recompute_tokens"]]


def test_kv_restatement_prefill_equals_reference(golden):
    d = golden["small_model"]
    m = _small_model(d)
    prompt = [int(t) for t in d["prompt"]]
    eng = KVGolden(m, kv="fp32")
    np.testing.assert_array_equal(eng.prefill(prompt), d["prompt_logits"][-1])
    # int8 KV: close to the fp32-cache logits, cache holds int8 rows
    e8 = KVGolden(m, kv="int8")
    lg = e8.prefill(prompt)
    ref = d["prompt_logits"][-1]
    assert np.max(np.abs(lg - ref)) < 0.05 * np.max(np.abs(ref))
    assert e8.k_cache.dtype == np.int8 and np.abs(e8.k_cache[:, :, :len(prompt)]).max() == 127


def test_kv_decode_matches_recompute_first_steps(golden):
    """With an fp32 cache the first decode step sees the same K/V rows as the
    recompute path; only activation-scale grouping differs, so logits agree
    closely and the greedy tokens match on this model."""
    d = golden["small_model"]
    m = _small_model(d)
    prompt = [int(t) for t in d["prompt"]]
    eng = KVGolden(m, kv="fp32")
    toks, reason, err = eng.generate(prompt, 6, eos_id=-1)
    assert err == 0 and reason == 2 and len(toks) == 6
    assert toks[0] == int(d["recompute_tokens"][0])


def test_config0_prefill_matches_reference(golden):
    if "config0" not in golden:
        pytest.skip("config0 fixture not generated")
    d = golden["config0"]
    m = W.quantize_archive(W.random_archive(int(d["seed"]), 1), "tensor")
    prompt = [int(t) for t in d["prompt"]]
    eng = KVGolden(m, kv="fp32")
    np.testing.assert_array_equal(eng.prefill(prompt), d["first_logits"])
    cos, sin = G.build_rope_cache(2048, 64, m.cfg["rope_theta"])
    assert G.generate_recompute(prompt, m, cos, sin, len(d["recompute_tokens"])) == \
        [int(t) for t in d["recompute_tokens"]]


def test_sim_kats(golden):
    d = golden["kat_sim"]
    # 64x64 GEMV KAT, W stored [N][K] (model/gen_test_vectors.py:15-32)
    np.testing.assert_array_equal(G.int8_matmul(d["gemv_w_nk"], d["gemv_x"][:, None])[:, 0],
                                  d["gemv_expected"])
    for k in (16, 64):
        x_q, w1, w2 = d[f"k{k}_x_q"], d[f"k{k}_W1_q"], d[f"k{k}_W2_q"]
        sx, s1, s2, sy2 = d[f"k{k}_scales"]
        y1 = G.int8_matmul(w1, x_q[:, None])[:, 0]
        np.testing.assert_array_equal(y1, d[f"k{k}_y1_int"])
        y1d = G.dequantize_int32(y1, s1, sx)
        y2q, s = G.quantize_int8(np.maximum(0, y1d))
        np.testing.assert_array_equal(y2q, d[f"k{k}_y2_q"])
        # scales.txt was written by an older NumPy (float64 scalar promotion);
        # the printed scale agrees to float32 precision, the bytes exactly.
        assert abs(s - sy2) <= 1e-6 * sy2
        np.testing.assert_array_equal(G.int8_matmul(w2, y2q[:, None])[:, 0], d[f"k{k}_y_expected"])


def test_contract_helpers(golden):
    d = golden["contract"]
    assert [C.q16_16_from_float(v) for v in d["q16_in"]] == list(d["q16_out"])
    assert [C.q16_16_signed_from_float(v) for v in d["q16s_in"]] == list(d["q16s_out"])
    np.testing.assert_array_equal(C.round_q16_16_sum_to_int8(d["rnd_in"]), d["rnd_out"])
    np.testing.assert_array_equal(C.rope_int8(d["rope_q"], d["rope_cos_q16"], d["rope_sin_q16"]),
                                  d["rope_q_out"])
    np.testing.assert_array_equal(C.rope_int8(d["rope_k"], d["rope_cos_q16"], d["rope_sin_q16"]),
                                  d["rope_k_out"])
    # RTL requantize vs the exporter's float-quantized expectation: the Q16.16
    # multiplier keeps 16 fractional bits, so the two agree to within 1 LSB.
    r = C.requantize_q16(d["req_acc"], d["req_mult_q16"])
    assert np.abs(r.astype(int) - d["req_float_expected"].astype(int)).max() <= 1


def test_requantize_rule_edges():
    acc = np.array([0, 1, -1, 32768, -32768, 98304, -98304, 2**31 - 1, -2**31], np.int64)
    # multiplier 1.0: exact passthrough then clamp
    np.testing.assert_array_equal(C.requantize_q16(acc, 65536),
                                  np.clip(acc, -127, 127).astype(np.int8))
    # multiplier 0.5: half-way cases go to even
    np.testing.assert_array_equal(C.requantize_q16(np.array([1, 3, 5, -1, -3]), 32768),
                                  np.array([0, 2, 2, 0, -2], np.int8))
    np.testing.assert_array_equal(C.requantize_q16(np.array([-5, 5]), 65536, nonnegative_only=True),
                                  np.array([0, 5], np.int8))


def test_stop_priority_and_addresses():
    assert C.stop_decision(True, True, 2, 0, 1, 2) == (True, 3)
    assert C.stop_decision(False, True, 2, 0, 1, 2) == (True, 1)
    assert C.stop_decision(False, True, 5, 0, 1, 2) == (True, 2)
    assert C.stop_decision(False, True, 5, 3, 0, 2) == (False, 0)
    assert C.kv_row_address(0x1000, 1, 2, 3) == 0x1000 + (((1 * 4 + 2) * 2048 + 3) << 6)
    assert C.status_word(False, True, False, True, 1, 0) == 0b1_1010


def test_analysis_fixture_float_and_int8_layers(golden):
    """The reference's run_analysis dump (tests/golden/analysis.npz, made by
    the reference itself): the oracle's float32 layer and INT8 golden layer
    reproduce its layer-0 arrays bit for bit, and its reported layer-0 MAE."""
    from oracle import weights as W
    d = golden["analysis"]
    arc = W.random_archive(int(d["seed"]), int(d["layers"]), W.small_dims(), gamma_one=False)
    w = W.ArchiveWeights(arc)
    cfg = w.cfg
    ids = [int(t) for t in d["token_ids"]]
    cos, sin = G.build_rope_cache(cfg["max_position_embeddings"], cfg["head_dim"], cfg["rope_theta"])
    x = w.embed(ids).astype(np.float32)
    ref_out = G.reference_decoder_layer(x, w.layer(0), cfg, cos, sin)
    np.testing.assert_array_equal(ref_out, d["dump__reference_layer_out_fp"])
    qm = W.quantize_archive(arc, "tensor")
    mix_out = G.decoder_layer_mixed(x, qm.layers[0], cfg, cos, sin)
    np.testing.assert_array_equal(mix_out, d["dump__mixed_layer_out_fp"])
    mae = float(np.abs(mix_out - ref_out).mean())
    assert f"isolated MAE={mae:.6f}" in str(d["summary"][3])


def test_contract_mode_wrappers_match_exporter(golden):
    """oracle/contract.py's fixed-point wrapper chain reproduces the
    exporter's own RMSNorm / SiLU / softmax / residual-add cases
    (tests/golden/contract_mode.npz, written by the exporter's build_*_case
    functions) bit for bit."""
    from oracle import contract as K
    d = golden["contract_mode"]
    for m in ("prefill", "decode"):
        y16, yq, yfp = K.rmsnorm_contract(d[f"rms_{m}_x_q"], d[f"rms_{m}_in_q16"], d[f"rms_{m}_gamma_q16"],
                                          float(d["rms_eps"]), d[f"rms_{m}_out_q16"])
        np.testing.assert_array_equal(yfp, d[f"rms_{m}_y_fp"])
        np.testing.assert_array_equal(y16, d[f"rms_{m}_y_q16"])
        np.testing.assert_array_equal(yq, d[f"rms_{m}_y_q"])
        y16, yq, yfp = K.silu_contract(d[f"silu_{m}_x_q"], d[f"silu_{m}_in_q16"], d[f"silu_{m}_out_q16"])
        np.testing.assert_array_equal(yfp, d[f"silu_{m}_y_fp"])
        np.testing.assert_array_equal(y16, d[f"silu_{m}_y_q16"])
        np.testing.assert_array_equal(yq, d[f"silu_{m}_y_q"])
        n = int(d[f"sm_{m}_rows"])
        p16, pq, pfp = K.softmax_contract(d[f"sm_{m}_score"][:n], d[f"sm_{m}_scale_q16"])
        np.testing.assert_array_equal(pfp, d[f"sm_{m}_prob_fp"][:n])
        np.testing.assert_array_equal(p16, d[f"sm_{m}_prob_q16"][:n])
        np.testing.assert_array_equal(pq, d[f"sm_{m}_prob_q"][:n])
    np.testing.assert_array_equal(K.residual_add_i32(d["res_a"], d["res_b"]), d["res_sum"])
    big = np.array([2**31 - 5, -2**31 + 3], np.int64)
    np.testing.assert_array_equal(K.residual_add_i32(big.astype(np.int32), np.array([10, -10], np.int32)),
                                  np.array([-2**31 + 5, 2**31 - 7], np.int64).astype(np.int32))
