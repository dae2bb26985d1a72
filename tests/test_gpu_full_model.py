"""The benchmark configurations end to end at full size (GPU): the 22-layer
TinyLlama (random per-output-channel INT8 weights, N(0, 0.02) before
quantization) against the KV-cached oracle with an exact INT8 matmul.

* batch 1, 128-token prompt, 32 greedy tokens through the
  persistent single-sequence decode kernel; prefill and teacher-forced
  decode logits.
* 64 sequences with 512-token prompts and 16 greedy steps on the
  batched tcgen05 decode path; 4 of the 64 sequences checked.
* 2048-token prompts on the persistent tcgen05 GEMMs and the
  tcgen05 prefill attention: last-row logits, and a two-sequence batch.

Tolerance. Every activation of the reference's pipeline is re-quantized to
INT8, so any float difference of ~1e-6 (a different attention summation
order) turns into 1-LSB flips that propagate through 22 layers: swapping
only the reference's float64 attention for float32 moves its own logits by
~8% (oracle/golden.py attention_core_f32; 7.7% at 128 tokens, 8.4% at 512
measured on this model). A fixed 1e-3 bound on 22-layer logits is therefore
below the reference's own numerical noise. Each check here holds the
engine's logits within max(1e-3, 3 x the distance between the oracle and
the oracle with its attention perturbed at the kernels' stated accuracy) of
the float64 oracle, measured on the same input and step
(helpers.oracle_run); greedy ids must agree except where the oracle's top-2
logits are closer than that bound. Op-level exactness (accumulators,
quantization, K/V bytes at every layer) is proven in test_gpu_layer.py;
layer-0 K/V bytes are exact here.
"""

import numpy as np
import pytest

from helpers import oracle_run, rel_err, to_engine_model, tokens_match_modulo_ties

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


@pytest.fixture(scope="module")
def tiny22(gpu, tinyllama22):
    return tinyllama22


def test_config2_batch1_decode(pkg, tiny22):
    qm, mm = tiny22
    eng = pkg.Engine(qm.cfg, max_batch=1, max_prefill_tokens=128)
    eng.load(to_engine_model(pkg, qm))
    prompt = [int(t) for t in np.random.default_rng(20).integers(0, 32000, 128)]
    toks, st = eng.generate(prompt, 32)
    assert st["generated_count"] == 32 and st["stop_reason"] == 2
    ref, ref_logits, bounds, ora = oracle_run(qm, prompt, 32, mm)
    assert tokens_match_modulo_ties(toks, ref, ref_logits, bounds), (toks, ref)
    k, v, _, _ = eng.read_kv(0, 128)
    np.testing.assert_array_equal(k, ora.k_cache[0, :, :128])
    np.testing.assert_array_equal(v, ora.v_cache[0, :, :128])
    lg = eng.prefill_logits(prompt)
    assert rel_err(lg, ref_logits[0]) <= bounds[0], (rel_err(lg, ref_logits[0]), bounds[0])
    for i in range(8):  # teacher-forced decode steps on the oracle's ids
        lg = eng.decode_logits(ref[i])
        assert rel_err(lg, ref_logits[i + 1]) <= bounds[i + 1], (i, rel_err(lg, ref_logits[i + 1]), bounds[i + 1])
    eng.close()


def test_config3_batch64_decode(pkg, tiny22):
    qm, mm = tiny22
    eng = pkg.Engine(qm.cfg, max_batch=64, max_prefill_tokens=64 * 512)
    eng.load(to_engine_model(pkg, qm))
    prompts = np.random.default_rng(21).integers(0, 32000, (64, 512)).astype(np.uint32)
    outs, sts = eng.generate_batch(prompts, 16)
    assert pkg.shim.load_library().tl_device_error() == 0
    assert all(s["generated_count"] == 16 for s in sts)
    for i in (0, 21, 42, 63):
        ref, ref_logits, bounds, ora = oracle_run(qm, [int(t) for t in prompts[i]], 16, mm)
        assert tokens_match_modulo_ties(outs[i], ref, ref_logits, bounds), (i, outs[i], ref)
        k, v, _, _ = eng.read_kv(0, 512, slot=i)
        np.testing.assert_array_equal(k, ora.k_cache[0, :, :512])
        np.testing.assert_array_equal(v, ora.v_cache[0, :, :512])
    eng.close()


def test_config4_long_prompt_prefill(pkg, tiny22):
    qm, mm = tiny22
    eng = pkg.Engine(qm.cfg, max_batch=2, max_prefill_tokens=2 * 2048)
    eng.load(to_engine_model(pkg, qm))
    prompts = np.random.default_rng(22).integers(0, 32000, (2, 2048)).astype(np.uint32)
    ref, ref_logits, bounds, ora = oracle_run(qm, [int(t) for t in prompts[1]], 1, mm)
    lg = eng.prefill_logits(prompts[1])
    assert rel_err(lg, ref_logits[0]) <= bounds[0], (rel_err(lg, ref_logits[0]), bounds[0])
    k, v, _, _ = eng.read_kv(0, 2048)
    np.testing.assert_array_equal(k, ora.k_cache[0])
    np.testing.assert_array_equal(v, ora.v_cache[0])
    # two sequences in one batched prefill (4096 rows): sequence 1 in slot 1
    outs, _ = eng.generate_batch(prompts, 1)
    assert pkg.shim.load_library().tl_device_error() == 0
    assert tokens_match_modulo_ties(outs[1], ref, ref_logits, bounds)
    k, v, _, _ = eng.read_kv(0, 2048, slot=1)
    np.testing.assert_array_equal(k, ora.k_cache[0])
    np.testing.assert_array_equal(v, ora.v_cache[0])
    eng.close()
