"""Single decoder layers on caller-given activations (GPU): the C ABI's
tl_decoder_layer / tl_decode_layer and the shim's reference-shaped operator
API, checked op by op (tests/layer_checks.py).

Two feeds:
* teacher forcing: layer l gets the ORACLE's layer-l input, so the exact
  prefix (RMSNorm, INT8 input, q/k/v accumulators) and the layer's INT8 K/V
  bytes are compared with the oracle's own values at every layer;
* self-chaining: layer l gets the engine's own layer-(l-1) output, which is
  what the production prefill / decode step computes; the chain's last hidden
  state (prefill) and the K/V rows of every layer (decode) must equal the
  production path's bit for bit, so the op-by-op checks of the chain cover
  the production kernels.
In both, every op is compared with the oracle op applied to the engine's own
inputs of that op: exact for integer work, RMSNorm, quantization, dequant and
residual adds; attention within 1e-5 and SiLU*up within 1e-6.

Why not whole-model logits at 1e-3: the reference's numerics re-quantize
every activation to INT8, so a 1e-6 float difference anywhere becomes a
1-LSB flip that propagates. Replacing only the reference's float64 attention
by float32 moves its own 22-layer logits by ~8% (measured: 7.7% at 128
tokens, 8.4% at 512); test_gpu_full_model.py bounds the engine end to end
relative to that measured sensitivity.
"""

import numpy as np
import pytest

from oracle import golden as G
from oracle import weights as W
from oracle.kv_golden import KVGolden

from helpers import FP_RTOL, rel_err, small_model, to_engine_model
from layer_checks import check_kv, check_layer_ops, check_layer_prefix

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def run_prefill_chain(eng, qm, ora, x, teacher: bool, slot=0, every=True, tag=""):
    """All layers of a one-sequence prefill through tl_decoder_layer; returns
    the engine's last layer output (self-chained) or the oracle's."""
    for li in range(len(qm.layers)):
        out_e, cap = eng.decoder_layer(li, x, slot=slot, capture=every)
        out_o, cap_o = ora.layer_capture(li, x)
        check_layer_prefix(cap, cap_o, f"{tag} layer {li}")
        check_kv(eng, ora, li, x.shape[0], slot=slot, tag=tag)
        check_layer_ops(cap, x, out_e, qm.layers[li], qm.cfg, cap_o["attended"], per_row=False,
                        tag=f"{tag} layer {li}")
        if teacher:
            assert rel_err(out_e, out_o) <= 5e-2, (tag, li, rel_err(out_e, out_o))
        x = out_o if teacher else out_e
        yield li, cap, cap_o
    run_prefill_chain.last = x


def test_decoder_layer_small_every_layer(pkg, gpu):
    """2-layer scaled model, 37-row prompt, every capture field including the
    score and probability windows, teacher forced."""
    qm = small_model(5, 2)
    eng = pkg.Engine(qm.cfg, max_batch=2, max_prefill_tokens=64)
    eng.load(to_engine_model(pkg, qm))
    ora = KVGolden(qm, kv="int8", matmul=G.ExactMatmul())
    ids = np.random.default_rng(6).integers(0, qm.cfg["vocab_size"], 37)
    x = qm.embed[ids].astype(np.float32)
    every = [n for n, _, _ in pkg.shim.CAPTURE_FIELDS]
    c = qm.cfg
    for li, cap, cap_o in run_prefill_chain(eng, qm, ora, x, True, slot=1, every=every, tag="small"):
        kd, _ = ora.dequantized_kv(li, 37)
        sc = (cap_o["q_rot"] @ G.repeat_kv(kd, c["num_key_value_groups"]).transpose(0, 2, 1)) * c["attn_scale"]
        sc[:, ~G.causal_mask(37)] = G.MASK_FILL
        pr = G.softmax(sc)
        tri = np.broadcast_to(G.causal_mask(37), sc.shape)
        assert np.max(np.abs(cap["scores"][tri] - sc[tri])) <= 1e-5 * np.max(np.abs(sc[tri]))
        assert np.all(cap["scores"][~tri] == np.float32(G.MASK_FILL))
        assert np.max(np.abs(cap["probs"] - pr)) <= 1e-6
    eng.close()


def test_decoder_layer_tinyllama_22_layers_teacher_forced(pkg, gpu, tinyllama22):
    """Full 22-layer TinyLlama (random per-channel INT8 weights), 48-token
    prompt, every layer fed the oracle's input for that layer: the exact
    prefix and the INT8 K/V cache of all 22 layers equal the oracle's, every
    op checks against the oracle on the engine's own inputs."""
    qm, mm = tinyllama22
    eng = pkg.Engine(qm.cfg, max_batch=1, max_prefill_tokens=64)
    eng.load(to_engine_model(pkg, qm))
    ora = KVGolden(qm, kv="int8", matmul=mm)
    ids = np.random.default_rng(7).integers(0, qm.cfg["vocab_size"], 48)
    for _ in run_prefill_chain(eng, qm, ora, qm.embed[ids].astype(np.float32), True, tag="tf22"):
        pass
    for li in range(22):
        check_kv(eng, ora, li, 48, tag="tf22 after all layers")
    eng.close()


def test_prefill_chain_equals_production(pkg, gpu, tinyllama22):
    """Self-chained 22-layer prefill (each layer fed the engine's own previous
    output, every op checked), 96-token prompt: the chain's K/V bytes of every
    layer and its final RMSNorm output equal the production prefill's
    (tl_forward_logits) bit for bit, and the production logits are the exact
    INT8 LM head of that hidden state."""
    qm, mm = tinyllama22
    eng = pkg.Engine(qm.cfg, max_batch=1, max_prefill_tokens=128)
    eng.load(to_engine_model(pkg, qm))
    ids = [int(t) for t in np.random.default_rng(8).integers(0, qm.cfg["vocab_size"], 96)]
    ora = KVGolden(qm, kv="int8", matmul=mm)
    for _ in run_prefill_chain(eng, qm, ora, qm.embed[np.asarray(ids)].astype(np.float32), False, tag="chain"):
        pass
    x_last = run_prefill_chain.last
    kv_chain = [eng.read_kv(li, 96) for li in range(22)]
    hidden = eng.forward_logits(ids, hidden=True)     # production prefill (overwrites the cache)
    for li in range(22):
        k, v, ks, vs = eng.read_kv(li, 96)
        np.testing.assert_array_equal(k, kv_chain[li][0], err_msg=f"layer {li} K: chain vs production")
        np.testing.assert_array_equal(v, kv_chain[li][1], err_msg=f"layer {li} V: chain vs production")
    want_h = G.rms_norm(x_last, qm.final_norm, qm.cfg["rms_norm_eps"])
    np.testing.assert_array_equal(hidden, want_h)
    logits = eng.forward_logits(ids)
    hq, sh = G.quantize_int8(want_h)
    np.testing.assert_array_equal(logits, G.dequantize_int32(G.int8_matmul(hq, qm.lm_head.w_q), sh,
                                                             qm.lm_head.scale))
    last = eng.prefill_logits(ids)
    np.testing.assert_array_equal(last, logits[-1])
    eng.close()


def test_decode_layer_chain_64_rows(pkg, gpu, tinyllama22):
    """configs[3] decode at full size, op by op: 64 sequences prefilled with
    512-token prompts and one production decode step (appending position
    512); then the same step re-run layer by layer through tl_decode_layer
    on the tcgen05 decode kernels, each layer fed the engine's own output.
    Checked: every op of 4 rows against the oracle (whose cache holds the
    engine's prompt K/V), the appended INT8 K/V row of every layer against
    the oracle's (exact) and against the production step's (bit for bit)."""
    qm, mm = tinyllama22
    eng = pkg.Engine(qm.cfg, max_batch=64, max_prefill_tokens=64 * 512)
    eng.load(to_engine_model(pkg, qm))
    prompts = np.random.default_rng(9).integers(0, 32000, (64, 512)).astype(np.uint32)
    outs, _ = eng.generate_batch(prompts, 2)
    checked = (0, 21, 42, 63)
    oras, prod = {}, {}
    for i in checked:
        ora = KVGolden(qm, kv="int8", matmul=mm)
        prod[i] = []
        for li in range(22):
            k, v, ks, vs = eng.read_kv(li, 513, slot=i)
            ora.k_cache[li, :, :512] = k[:, :512]
            ora.v_cache[li, :, :512] = v[:, :512]
            ora.k_scale[li] = ks
            ora.v_scale[li] = vs
            prod[i].append((k[:, 512].copy(), v[:, 512].copy()))
        oras[i] = ora
    x = qm.embed[np.asarray([o[0] for o in outs])].astype(np.float32)
    for li in range(22):
        out_e, cap = eng.decode_layer(li, x, slots=np.arange(64), positions=np.full(64, 512), capture=True)
        for i in checked:
            _, cap_o = oras[i].layer_capture(li, x[i:i + 1], p0=512, prefill=False)
            check_layer_prefix(cap, cap_o, f"decode row {i} layer {li}", row=i)
            sub = {k: (v[i:i + 1] if np.ndim(v) == 2 else v[i:i + 1]) for k, v in cap.items()}
            check_layer_ops(sub, x[i:i + 1], out_e[i:i + 1], qm.layers[li], qm.cfg, cap_o["attended"],
                            per_row=True, tag=f"decode row {i} layer {li}")
            k, v, _, _ = eng.read_kv(li, 513, slot=i)
            np.testing.assert_array_equal(k[:, 512], oras[i].k_cache[li, :, 512], err_msg=f"row {i} layer {li} K")
            np.testing.assert_array_equal(v[:, 512], oras[i].v_cache[li, :, 512], err_msg=f"row {i} layer {li} V")
            np.testing.assert_array_equal(k[:, 512], prod[i][li][0], err_msg=f"row {i} layer {li} K vs production")
            np.testing.assert_array_equal(v[:, 512], prod[i][li][1], err_msg=f"row {i} layer {li} V vs production")
        x = out_e
    eng.close()


def test_decoder_layer_long_prompt_tensor_core_path(pkg, gpu):
    """TinyLlama widths at 700 rows: the projections run on the persistent
    tcgen05 GEMM and attention on the tcgen05 prefill kernel (several query
    tiles); teacher forced, one layer."""
    dims = W.small_dims(vocab=512, hidden=2048, ffn=5632, heads=32, kv_heads=4)
    qm = W.random_qmodel(77, 1, dims)
    eng = pkg.Engine(qm.cfg, max_batch=1, max_prefill_tokens=1024)
    eng.load(to_engine_model(pkg, qm))
    ora = KVGolden(qm, kv="int8", matmul=G.ExactMatmul())
    x = qm.embed[np.random.default_rng(8).integers(0, 512, 700)].astype(np.float32)
    for _ in run_prefill_chain(eng, qm, ora, x, True, tag="700 rows"):
        pass
    eng.close()


def test_decoder_layer_rejects_bad_calls(pkg, gpu):
    qm = small_model(5, 1)
    eng = pkg.Engine(qm.cfg, max_batch=1, max_prefill_tokens=64)
    eng.load(to_engine_model(pkg, qm))
    x = np.zeros((4, qm.cfg["hidden_size"]), np.float32)
    with pytest.raises(pkg.TLError) as e:
        eng.decoder_layer(1, x)          # layer out of range
    assert e.value.code == 17
    with pytest.raises(pkg.TLError) as e:
        eng.decoder_layer(0, x, slot=3)  # slot out of range
    assert e.value.code == 17
    with pytest.raises(pkg.TLError) as e:
        eng.decoder_layer(0, x[:0])      # no rows: bad descriptor
    assert e.value.code == 1
    with pytest.raises(ValueError):
        eng.decoder_layer(0, x[:, :8])
    eng.close()


REF_ATTN_KEYS = {"q_proj", "k_proj", "v_proj", "o_proj", "q_proj_fp", "k_proj_fp", "v_proj_fp"}
REF_FFN_KEYS = {"gate_proj", "up_proj", "down_proj", "gate_proj_fp", "up_proj_fp", "hidden_fp"}
REF_LIN_KEYS = {"input_scale", "weight_scale"}
REF_LIN_CAPTURE = {"input_fp", "input_q", "weight_fp", "weight_q", "accum_int32", "output_fp"}


def test_mixed_precision_decoder_layer_reference_api(pkg, gpu):
    """shim.mixed_precision_decoder_layer takes the reference's layer dict
    (float [in, out] weights, quantized per tensor as the bridge does) and
    returns the reference's (out, debug) structure
    (model/tinyllama_gemm_int8.py:136-281); values against the oracle."""
    arc = W.random_archive(9, 1, W.small_dims(), gamma_one=False)
    weights = W.ArchiveWeights(arc)
    qm = W.quantize_archive(arc, "tensor")
    x = qm.embed[np.random.default_rng(10).integers(0, 512, 21)].astype(np.float32)
    layer = weights.layer(0)
    out, dbg = pkg.mixed_precision_decoder_layer(x, layer, weights.cfg, None, None, capture_arrays=False)
    assert set(dbg) == {"attn_input_fp", "x_after_attn_fp", "ffn_input_fp", "attn", "ffn"}
    assert set(dbg["attn"]) == REF_ATTN_KEYS and set(dbg["ffn"]) == REF_FFN_KEYS
    assert set(dbg["attn"]["q_proj"]) == REF_LIN_KEYS
    out2, dbg2 = pkg.mixed_precision_decoder_layer(x, layer, weights.cfg, None, None, capture_arrays=True)
    np.testing.assert_array_equal(out, out2)
    assert set(dbg2["attn"]) == REF_ATTN_KEYS | {"scores_fp", "weights_fp", "attended_fp", "out_fp"}
    assert set(dbg2["ffn"]) == REF_FFN_KEYS | {"out_fp"}
    assert set(dbg2["attn"]["o_proj"]) == REF_LIN_KEYS | REF_LIN_CAPTURE
    assert "layer_out_fp" in dbg2
    ora = KVGolden(qm, kv="int8")
    ref_out, cap = ora.layer_capture(0, x)
    assert rel_err(out, ref_out) <= FP_RTOL
    q = dbg2["attn"]["q_proj"]
    np.testing.assert_array_equal(q["accum_int32"], cap["q_acc"])
    np.testing.assert_array_equal(q["input_q"], cap["qkv_input_q"])
    np.testing.assert_array_equal(q["weight_q"], qm.layers[0].q.w_q)
    _, s_ref = G.quantize_int8(x_norm := G.rms_norm(x, qm.layers[0].input_norm, qm.cfg["rms_norm_eps"]))
    assert q["input_scale"][0] == np.float32(s_ref)
    assert q["weight_scale"][0] == np.float32(qm.layers[0].q.scale[0])
    np.testing.assert_array_equal(dbg2["attn_input_fp"], x_norm)
    o = dbg2["attn"]["o_proj"]
    np.testing.assert_array_equal(o["accum_int32"], G.int8_matmul(o["input_q"], qm.layers[0].o.w_q))


def test_forward_mixed_all_rows(pkg, gpu):
    """shim.forward_mixed returns logits for every row ([S, vocab]) like the
    reference; quantize_lm_head=False multiplies the final hidden state by
    the float LM head."""
    arc = W.random_archive(12, 2, W.small_dims(), gamma_one=False)
    weights = W.ArchiveWeights(arc)
    qm = W.quantize_archive(arc, "tensor")
    ids = [int(t) for t in np.random.default_rng(13).integers(0, 512, 19)]
    lg = pkg.forward_mixed(ids, weights, None, None, 2, quantize_lm_head=True)
    assert lg.shape == (19, 512) and lg.dtype == np.float32
    ora = KVGolden(qm, kv="int8")
    x = qm.embed[np.asarray(ids)].astype(np.float32)
    for li in range(2):
        x = ora._layer(li, x, 0, True)
    hn = G.rms_norm(x, qm.final_norm, qm.cfg["rms_norm_eps"])
    ref, _, _, _ = G.linear_q(hn, qm.lm_head.w_q, qm.lm_head.scale)
    for r in range(19):
        assert rel_err(lg[r], ref[r]) <= FP_RTOL, (r, rel_err(lg[r], ref[r]))
    lf = pkg.forward_mixed(ids, weights, None, None, 2, quantize_lm_head=False)
    reff = hn @ weights.lm_head_w()
    assert lf.shape == (19, 512)
    assert rel_err(lf, reff) <= FP_RTOL
    with pytest.raises(ValueError):
        pkg.forward_mixed(ids, weights, None, None, 3)
