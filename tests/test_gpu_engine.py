"""Engine-level parity (GPU): prefill, decode, INT8 KV cache, generation and
the RTL stop contract, against the KV-cached oracle (oracle/kv_golden.py).

Tolerances: INT8 KV-cache bytes of layer 0 are bit-exact (every op feeding
them is exact); float blocks within 1e-3 relative; greedy ids identical
except where the oracle's top-2 logits are closer than that tolerance.
"""

import threading

import numpy as np
import pytest

from oracle import golden as G
from oracle import weights as W
from oracle.kv_golden import KVGolden

from helpers import FP_RTOL, rel_err, small_model, to_engine_model, tokens_match_modulo_ties

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


@pytest.fixture(scope="module")
def small(pkg, gpu):
    qm = small_model(7, 2)
    eng = pkg.Engine(qm.cfg, max_batch=4, max_prefill_tokens=2048 * 1)
    eng.load(to_engine_model(pkg, qm))
    yield qm, eng
    eng.close()


def oracle_generate(qm, prompt, n, eos=-1):
    ora = KVGolden(qm, kv="int8")
    logits = [ora.prefill(prompt)]
    toks = []
    for _ in range(n):
        t = G.argmax_first(logits[-1])
        toks.append(t)
        if t == eos or len(toks) == n:
            break
        logits.append(ora.decode(t))
    return toks, logits, ora


def test_prefill_logits_and_kv_cache(small):
    qm, eng = small
    prompt = list(np.random.default_rng(1).integers(0, qm.cfg["vocab_size"], 11))
    lg = eng.prefill_logits(prompt)
    ora = KVGolden(qm, kv="int8")
    ref = ora.prefill(prompt)
    assert rel_err(lg, ref) <= FP_RTOL, rel_err(lg, ref)
    k, v, ks, vs = eng.read_kv(0, len(prompt))
    np.testing.assert_array_equal(k, ora.k_cache[0, :, :len(prompt)])
    np.testing.assert_array_equal(v, ora.v_cache[0, :, :len(prompt)])
    np.testing.assert_array_equal(ks, ora.k_scale[0].astype(np.float32))
    np.testing.assert_array_equal(vs, ora.v_scale[0].astype(np.float32))
    # deeper layers: float-path differences may flip isolated INT8 values by 1
    k1, v1, _, _ = eng.read_kv(1, len(prompt))
    assert np.abs(k1.astype(int) - ora.k_cache[1, :, :len(prompt)]).max() <= 1
    assert np.mean(k1 != ora.k_cache[1, :, :len(prompt)]) < 0.01


def test_decode_teacher_forced(small):
    qm, eng = small
    prompt = list(np.random.default_rng(2).integers(0, qm.cfg["vocab_size"], 6))
    eng.prefill_logits(prompt)
    ora = KVGolden(qm, kv="int8")
    ora.prefill(prompt)
    feed = list(np.random.default_rng(3).integers(0, qm.cfg["vocab_size"], 8))
    for t in feed:
        lg = eng.decode_logits(t)
        ref = ora.decode(t)
        assert rel_err(lg, ref) <= FP_RTOL
    assert eng.position() == len(prompt) + len(feed)
    k, _, _, _ = eng.read_kv(0, ora.pos)
    np.testing.assert_array_equal(k, ora.k_cache[0, :, :ora.pos])


def test_generate_matches_oracle(small):
    qm, eng = small
    prompt = list(np.random.default_rng(4).integers(0, qm.cfg["vocab_size"], 9))
    toks, st = eng.generate(prompt, 12)
    ref, ref_logits, _ = oracle_generate(qm, prompt, 12)
    assert st["stop_reason"] == 2 and st["generated_count"] == 12
    assert tokens_match_modulo_ties(toks, ref, ref_logits)


def test_generate_batch_matches_single(small):
    qm, eng = small
    rng = np.random.default_rng(5)
    prompts = rng.integers(0, qm.cfg["vocab_size"], (3, 7)).astype(np.uint32)
    outs, sts = eng.generate_batch(prompts, 6)
    for i in range(3):
        ref, ref_logits, _ = oracle_generate(qm, list(prompts[i]), 6)
        assert tokens_match_modulo_ties(outs[i], ref, ref_logits)
        assert sts[i]["stop_reason"] == 2


def test_batched_tensor_core_path(pkg, gpu):
    """20 sequences: prefill (140 rows) and every decode step run on the
    tcgen05 GEMMs with split-K cluster reductions; each sequence must follow
    its own oracle."""
    qm = small_model(11, 2)
    eng = pkg.Engine(qm.cfg, max_batch=20, max_prefill_tokens=20 * 7)
    eng.load(to_engine_model(pkg, qm))
    rng = np.random.default_rng(12)
    prompts = rng.integers(0, qm.cfg["vocab_size"], (20, 7)).astype(np.uint32)
    outs, sts = eng.generate_batch(prompts, 6)
    assert pkg.shim.load_library().tl_device_error() == 0
    mism = 0
    for i in range(20):
        ref, ref_logits, _ = oracle_generate(qm, list(prompts[i]), 6)
        assert sts[i]["stop_reason"] == 2 and sts[i]["generated_count"] == 6
        assert tokens_match_modulo_ties(outs[i], ref, ref_logits), (i, outs[i], ref)
        mism += outs[i] != ref
    k, _, _, _ = eng.read_kv(0, 7, slot=5)
    ora = KVGolden(qm, kv="int8")
    ora.prefill(list(prompts[5]))
    np.testing.assert_array_equal(k, ora.k_cache[0, :, :7])
    eng.close()


def test_uneven_row_groups(pkg, gpu):
    """49 sequences: the decode step runs them as two concurrent row groups of
    24 and 25 rows (two streams, one LM head over all 49); the first and last
    sequence of each group must follow its own oracle; so must a 16-row
    batch, which runs as one group."""
    qm = small_model(13, 2)
    eng = pkg.Engine(qm.cfg, max_batch=49, max_prefill_tokens=49 * 6)
    eng.load(to_engine_model(pkg, qm))
    assert eng.decode_row_groups(49) == 2 and eng.decode_row_groups(47) == 1 and eng.decode_row_groups(16) == 1
    rng = np.random.default_rng(14)
    prompts = rng.integers(0, qm.cfg["vocab_size"], (49, 6)).astype(np.uint32)
    outs, sts = eng.generate_batch(prompts, 5)
    assert pkg.shim.load_library().tl_device_error() == 0
    for i in (0, 23, 24, 48):
        ref, ref_logits, _ = oracle_generate(qm, list(prompts[i]), 5)
        assert sts[i]["stop_reason"] == 2 and sts[i]["generated_count"] == 5
        assert tokens_match_modulo_ties(outs[i], ref, ref_logits), (i, outs[i], ref)
    outs16, _ = eng.generate_batch(prompts[:16], 5)
    for i in (0, 15):
        ref, ref_logits, _ = oracle_generate(qm, list(prompts[i]), 5)
        assert tokens_match_modulo_ties(outs16[i], ref, ref_logits), (i, outs16[i], ref)
    eng.close()


def test_small_batches_on_tensor_cores(pkg, gpu):
    """3, 4, 8 and 15 sequences: batched decode steps of 2 or more rows run
    on the tcgen05 GEMMs with most of each 32-token tile empty (the same
    kernels as the large batches); the first and last sequence of each batch
    must follow its own oracle."""
    qm = small_model(17, 2)
    eng = pkg.Engine(qm.cfg, max_batch=15, max_prefill_tokens=15 * 6)
    eng.load(to_engine_model(pkg, qm))
    rng = np.random.default_rng(18)
    prompts = rng.integers(0, qm.cfg["vocab_size"], (15, 6)).astype(np.uint32)
    for n in (3, 4, 8, 15):
        outs, sts = eng.generate_batch(prompts[:n], 5)
        assert pkg.shim.load_library().tl_device_error() == 0
        for i in (0, n - 1):
            ref, ref_logits, _ = oracle_generate(qm, list(prompts[i]), 5)
            assert sts[i]["stop_reason"] == 2 and sts[i]["generated_count"] == 5
            assert tokens_match_modulo_ties(outs[i], ref, ref_logits), (n, i, outs[i], ref)
    eng.close()


def test_batched_decode_full_width(pkg, gpu):
    """TinyLlama widths (hidden 2048, FFN 5632, 32/4 heads; 1 layer, vocab
    2048) at 16 sequences: the batched decode step runs its tcgen05 GEMMs and
    the warp-per-row RMSNorm/quantize kernels at their production shapes;
    every sequence must follow its own oracle, layer-0 KV bytes exact."""
    dims = W.small_dims(vocab=2048, hidden=2048, ffn=5632, heads=32, kv_heads=4)
    qm = W.quantize_archive(W.random_archive(21, 1, dims, gamma_one=False), "channel")
    eng = pkg.Engine(qm.cfg, max_batch=16, max_prefill_tokens=16 * 6)
    eng.load(to_engine_model(pkg, qm))
    rng = np.random.default_rng(22)
    prompts = rng.integers(0, dims["vocab_size"], (16, 6)).astype(np.uint32)
    outs, sts = eng.generate_batch(prompts, 4)
    assert pkg.shim.load_library().tl_device_error() == 0
    for i in range(16):
        ref, ref_logits, ora = oracle_generate(qm, list(prompts[i]), 4)
        assert sts[i]["generated_count"] == 4
        assert tokens_match_modulo_ties(outs[i], ref, ref_logits), (i, outs[i], ref)
        if outs[i] == ref:
            n = 6 + len(ref) - 1
            k, v, _, _ = eng.read_kv(0, n, slot=i)
            np.testing.assert_array_equal(k, ora.k_cache[0, :, :n])
            np.testing.assert_array_equal(v, ora.v_cache[0, :, :n])
    eng.close()


def test_batched_decode_full_vocab_argmax(pkg, gpu):
    """Vocabulary 32000 at 16 sequences: the LM head of each decode step runs
    as 250 unsplit tcgen05 tiles with the greedy argmax fused into the
    epilogue (per-warp key exchange, per-CTA and global 64-bit maxima). The
    LM-head row of t2, the oracle's token from sequence 0's first decode
    step, is copied to another id d in a different tile, so at that step the
    two logits tie exactly and the lower id must be emitted."""
    import dataclasses
    dims = W.small_dims(vocab=32000)
    qm = W.quantize_archive(W.random_archive(31, 1, dims, gamma_one=False), "channel")
    rng = np.random.default_rng(32)
    prompts = rng.integers(0, dims["vocab_size"], (16, 5)).astype(np.uint32)
    ref0, _, _ = oracle_generate(qm, list(prompts[0]), 2)
    t1, t2 = ref0
    d = next(c for c in ((t2 + 16000) % 32000, (t2 + 9000) % 32000) if c != t1)
    w = qm.lm_head.w_q.copy()
    sc = qm.lm_head.scale.copy()
    w[:, d] = w[:, t2]
    sc[d] = sc[t2]
    qm = dataclasses.replace(qm, lm_head=W.QLinear(w, sc))
    eng = pkg.Engine(qm.cfg, max_batch=16, max_prefill_tokens=16 * 5)
    eng.load(to_engine_model(pkg, qm))
    outs, sts = eng.generate_batch(prompts, 4)
    assert pkg.shim.load_library().tl_device_error() == 0
    for i in range(16):
        ref, ref_logits, _ = oracle_generate(qm, list(prompts[i]), 4)
        assert sts[i]["generated_count"] == 4
        assert tokens_match_modulo_ties(outs[i], ref, ref_logits), (i, outs[i], ref)
    ref, ref_logits, _ = oracle_generate(qm, list(prompts[0]), 2)
    lg = np.asarray(ref_logits[1])
    assert lg[d] == lg[t2] and lg.argmax() == min(d, t2)  # the tie is real and on top
    assert outs[0][:2] == [t1, min(d, t2)], (outs[0], t1, t2, d)
    eng.close()


def test_long_prompts_multi_tile_prefill(pkg, gpu):
    """Prompts longer than one 64-position attention tile (ragged 150 and 130
    tokens): prefill logits and layer-0 KV bytes of one sequence, then a
    two-sequence batch through generate_batch, each against its oracle."""
    qm = small_model(13, 2)
    eng = pkg.Engine(qm.cfg, max_batch=2, max_prefill_tokens=2 * 150)
    eng.load(to_engine_model(pkg, qm))
    rng = np.random.default_rng(14)
    prompt = list(rng.integers(0, qm.cfg["vocab_size"], 150))
    lg = eng.prefill_logits(prompt)
    ora = KVGolden(qm, kv="int8")
    ref = ora.prefill(prompt)
    assert rel_err(lg, ref) <= FP_RTOL, rel_err(lg, ref)
    k, v, _, _ = eng.read_kv(0, len(prompt))
    np.testing.assert_array_equal(k, ora.k_cache[0, :, :len(prompt)])
    np.testing.assert_array_equal(v, ora.v_cache[0, :, :len(prompt)])
    prompts = rng.integers(0, qm.cfg["vocab_size"], (2, 130)).astype(np.uint32)
    outs, sts = eng.generate_batch(prompts, 4)
    for i in range(2):
        ref_t, ref_logits, _ = oracle_generate(qm, list(prompts[i]), 4)
        assert tokens_match_modulo_ties(outs[i], ref_t, ref_logits), (i, outs[i], ref_t)
    eng.close()


def test_single_sequence_long_context(pkg, gpu):
    """Batch-1 decode (the persistent single-sequence step) past 256 cached
    positions, where the attention partials of more than eight 32-position
    chunks are merged in several load rounds: tokens and logits follow the
    oracle; layer-0 KV bytes exact."""
    qm = small_model(17, 2)
    eng = pkg.Engine(qm.cfg, max_batch=1, max_prefill_tokens=320)
    eng.load(to_engine_model(pkg, qm))
    prompt = list(np.random.default_rng(18).integers(0, qm.cfg["vocab_size"], 300))
    toks, st = eng.generate(prompt, 6)
    ref, ref_logits, ora = oracle_generate(qm, prompt, 6)
    assert st["generated_count"] == 6
    assert tokens_match_modulo_ties(toks, ref, ref_logits), (toks, ref)
    if toks == ref:
        n = len(prompt) + len(ref) - 1
        k, v, _, _ = eng.read_kv(0, n)
        np.testing.assert_array_equal(k, ora.k_cache[0, :, :n])
        np.testing.assert_array_equal(v, ora.v_cache[0, :, :n])
    eng.close()


def test_stop_contract(small):
    qm, eng = small
    prompt = list(np.random.default_rng(6).integers(0, qm.cfg["vocab_size"], 5))
    ref, _, _ = oracle_generate(qm, prompt, 4)
    # EOS on the first token: one token, reason EOS
    toks, st = eng.generate(prompt, 10, eos_id=ref[0])
    assert toks == [ref[0]] and st["stop_reason"] == 1
    # EOS wins over MAX when both hit on the same token
    toks, st = eng.generate(prompt, 1, eos_id=ref[0])
    assert st["stop_reason"] == 1
    # prefill-only launch
    toks, st = eng.generate(prompt, 0)
    assert toks == [] and st["stop_reason"] == 0 and st["error_code"] == 0
    assert eng.position() == len(prompt)
    # empty prompt in prefill mode: bad descriptor (prefill_decode_controller.sv:85-88)
    toks, st = eng.generate([], 3, raise_on_error=False)
    assert st["return_code"] == 1 and st["error_code"] == 1
    # unsupported mode
    _, st = eng.generate(prompt, 3, mode=5, raise_on_error=False)
    assert st["return_code"] == 6


def test_decode_mode_continuation(small):
    qm, eng = small
    prompt = list(np.random.default_rng(8).integers(0, qm.cfg["vocab_size"], 5))
    first, _ = eng.generate(prompt, 3)
    more, st = eng.generate([], 4, mode=1)
    ref, ref_logits, _ = oracle_generate(qm, prompt, 7)
    assert tokens_match_modulo_ties(first + more, ref, ref_logits)
    assert st["generated_count"] == 4


def test_capacity_limit(pkg, gpu):
    qm = small_model(7, 1)
    cfg = dict(qm.cfg)
    cfg["max_position_embeddings"] = 64
    qm.cfg = cfg
    eng = pkg.Engine(cfg, max_batch=1)
    eng.load(to_engine_model(pkg, qm))
    prompt = list(np.random.default_rng(9).integers(0, cfg["vocab_size"], 62))
    toks, st = eng.generate(prompt, 10, raise_on_error=False)
    # tokens at positions 62 and 63 are processed; the third emitted token
    # would need position 64
    assert len(toks) == 3 and st["error_code"] == 17 and st["stop_reason"] == 4
    _, st = eng.generate(list(range(65)), 1, raise_on_error=False)
    assert st["return_code"] == 17
    eng.close()


def test_host_abort(pkg, gpu):
    qm = small_model(3, 8)
    eng = pkg.Engine(qm.cfg, max_batch=1)
    eng.load(to_engine_model(pkg, qm))
    prompt = [1, 2, 3, 4]
    res = {}

    def run():
        res["out"] = eng.generate(prompt, 2000, out_cap=2000)

    th = threading.Thread(target=run)
    th.start()
    import time
    time.sleep(0.05)
    eng.abort()
    th.join(timeout=120)
    toks, st = res["out"]
    assert st["stop_reason"] in (3, 2)
    if st["stop_reason"] == 3:
        assert 0 < len(toks) < 2000
    eng.close()


def test_config0_full_size(pkg, gpu, golden):
    """Benchmark config 0: one full-size TinyLlama layer, per-output-channel
    INT8 weights, 32-token prompt + 16 greedy decode steps."""
    qm = W.quantize_archive(W.random_archive(0, 1), "channel")
    eng = pkg.Engine(qm.cfg, max_batch=1)
    eng.load(to_engine_model(pkg, qm))
    prompt = [int(t) for t in np.random.default_rng(1).integers(0, 32000, 32)]
    lg = eng.prefill_logits(prompt)
    ora = KVGolden(qm, kv="int8")
    ref = ora.prefill(prompt)
    assert rel_err(lg, ref) <= FP_RTOL
    k, v, _, _ = eng.read_kv(0, 32)
    np.testing.assert_array_equal(k, ora.k_cache[0, :, :32])
    np.testing.assert_array_equal(v, ora.v_cache[0, :, :32])
    toks, st = eng.generate(prompt, 16)
    ref_toks, ref_logits, _ = oracle_generate(qm, prompt, 16)
    assert tokens_match_modulo_ties(toks, ref_toks, ref_logits)
    eng.close()


def test_reference_golden_first_token(pkg, gpu, golden):
    """Against the reference's own forward_mixed output (per-tensor weights,
    fixture made by the reference): the engine equals the INT8-KV oracle to
    1e-3, so its whole distance to the reference is the INT8 KV cache (which
    the reference does not have); the greedy token is the reference's."""
    if "config0" not in golden:
        pytest.skip("config0 fixture missing")
    d = golden["config0"]
    qm = W.quantize_archive(W.random_archive(int(d["seed"]), 1), "tensor")
    eng = pkg.Engine(qm.cfg, max_batch=1)
    eng.load(to_engine_model(pkg, qm))
    prompt = [int(t) for t in d["prompt"]]
    lg = eng.prefill_logits(prompt)
    ora = KVGolden(qm, kv="int8").prefill(prompt)
    assert rel_err(lg, ora) <= FP_RTOL
    ref = d["first_logits"]
    assert abs(rel_err(lg, ref) - rel_err(ora, ref)) <= FP_RTOL
    top2 = np.sort(ref)[-2:]
    if top2[1] - top2[0] > FP_RTOL * abs(top2[1]):
        assert int(np.argmax(lg)) == int(d["recompute_tokens"][0])
    eng.close()


def test_checkpoint_npz_generation(pkg, gpu, tmp_path):
    """A float16 weight archive in the reference's npz schema
    (model/tinyllama.py:292-382), read and quantized per output channel by
    load_checkpoint_npz, drives the engine: each sequence's greedy ids follow
    the oracle run on the oracle's quantization of the same arrays."""
    arc = W.random_archive(41, 2, W.small_dims(), gamma_one=False)
    arc = {k: (v.astype(np.float16) if k.startswith(("layer", "embed", "final", "lm_head")) else v)
           for k, v in arc.items()}
    path = tmp_path / "weights.npz"
    np.savez(path, **arc)
    model = pkg.load_checkpoint_npz(path)
    qm = W.quantize_archive(arc, "channel")
    eng = pkg.Engine(model.cfg, max_batch=4, max_prefill_tokens=4 * 8)
    eng.load(model)
    prompts = np.random.default_rng(42).integers(0, model.cfg["vocab_size"], (4, 8)).astype(np.uint32)
    outs, sts = eng.generate_batch(prompts, 5)
    assert pkg.shim.load_library().tl_device_error() == 0
    for i in range(4):
        ref, ref_logits, _ = oracle_generate(qm, list(prompts[i]), 5)
        assert sts[i]["generated_count"] == 5
        assert tokens_match_modulo_ties(outs[i], ref, ref_logits), (i, outs[i], ref)
    eng.close()
