"""Operator-level parity of the CUDA kernels against the oracle (GPU).

Integer results (INT32 accumulators, INT8 quantization, Q16.16 requantize)
must be bit-exact; RMSNorm is bit-exact as well because the kernel follows
NumPy's float32 reduction order.
"""

import numpy as np
import pytest

from oracle import contract as C
from oracle import golden as G

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return pkg.load_library()


def stream():
    return torch.cuda.current_stream().cuda_stream


_KEEP = []


def dev(a):
    """Device copy kept alive until the next test: passing a temporary's
    data_ptr() would let the caching allocator hand its block to the next
    argument before the kernel runs."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


@pytest.fixture(autouse=True)
def _release():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def gemm_gpu(lib, pkg, a, w_kn):
    m, k = a.shape
    n = w_kn.shape[1]
    wnk = dev(np.ascontiguousarray(w_kn.T))
    c = torch.empty((m, n), dtype=torch.int32, device="cuda")
    pkg.shim.check(lib.tl_gemm_i8(dev(a).data_ptr(), wnk.data_ptr(), c.data_ptr(), m, n, k, stream()), "gemm")
    return c.cpu().numpy()


@pytest.mark.parametrize("m,k,n", [(1, 64, 64), (1, 2048, 256), (3, 2048, 2048), (8, 5632, 2048),
                                   (17, 2048, 320), (32, 5632, 256), (1, 2048, 32000), (5, 704, 96),
                                   # tcgen05 path (m >= 16): tails in m, n and k, split-K clusters
                                   (16, 2048, 256), (64, 2048, 2560), (100, 704, 96), (300, 2048, 2048),
                                   (64, 5632, 2048), (48, 2048, 11264), (257, 256, 130), (64, 256, 512)])
def test_gemm_i8_bit_exact(lib, pkg, m, k, n):
    rng = np.random.default_rng(m * 131 + k + n)
    a = rng.integers(-127, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (k, n)).astype(np.int8)
    np.testing.assert_array_equal(gemm_gpu(lib, pkg, a, w), G.int8_matmul(a, w))


def test_gemm_extremes_and_kats(lib, pkg, golden):
    a = np.full((2, 5632), -127, np.int8)
    w = np.full((5632, 16), 127, np.int8)
    np.testing.assert_array_equal(gemm_gpu(lib, pkg, a, w), G.int8_matmul(a, w))
    d = golden["kat_sim"]
    got = gemm_gpu(lib, pkg, d["gemv_x"][None, :], np.ascontiguousarray(d["gemv_w_nk"].T))[0]
    np.testing.assert_array_equal(got, d["gemv_expected"])
    for k in (16, 64):
        y1 = gemm_gpu(lib, pkg, d[f"k{k}_x_q"][None, :], np.ascontiguousarray(d[f"k{k}_W1_q"].T))[0]
        np.testing.assert_array_equal(y1, d[f"k{k}_y1_int"])
        y = gemm_gpu(lib, pkg, d[f"k{k}_y2_q"][None, :], np.ascontiguousarray(d[f"k{k}_W2_q"].T))[0]
        np.testing.assert_array_equal(y, d[f"k{k}_y_expected"])


@pytest.mark.parametrize("per_col,nonneg", [(0, 0), (1, 0), (0, 1)])
def test_gemm_requant_bit_exact(lib, pkg, per_col, nonneg):
    rng = np.random.default_rng(10 + per_col + 2 * nonneg)
    m, k, n = 6, 2048, 512
    a = rng.integers(-127, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (k, n)).astype(np.int8)
    scales = rng.uniform(1e-4, 1e-2, n if per_col else 1)
    sq = np.array([C.q16_16_from_float(s) for s in scales], dtype=np.uint32)
    out = torch.empty((m, n), dtype=torch.int8, device="cuda")
    pkg.shim.check(lib.tl_gemm_i8_requant(dev(a).data_ptr(), dev(np.ascontiguousarray(w.T)).data_ptr(),
                                          dev(sq).data_ptr(), per_col, nonneg, out.data_ptr(), m, n, k,
                                          stream()), "requant")
    ref = C.requantize_q16(G.int8_matmul(a, w), sq[None, :] if per_col else sq[0], bool(nonneg))
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_quantize_int8_bit_exact(lib, pkg, golden):
    d = golden["quant_cases"]
    for key in ("q0", "q1", "q2", "q3", "q4", "qz", "qh"):
        x = np.atleast_2d(d[f"{key}_x"])
        q = torch.empty(x.shape, dtype=torch.int8, device="cuda")
        am = torch.empty(1, dtype=torch.float32, device="cuda")
        pkg.shim.check(lib.tl_quantize_int8(dev(x).data_ptr(), x.shape[0], x.shape[1], x.shape[0],
                                            q.data_ptr(), am.data_ptr(), stream()), "quantize")
        np.testing.assert_array_equal(q.cpu().numpy().reshape(d[f"{key}_q"].shape), d[f"{key}_q"], err_msg=key)
        peak = float(am.item())
        assert (1.0 if peak == 0.0 else peak / 127.0) == float(d[f"{key}_scale"]), key


def test_quantize_int8_adversarial_quotients(lib, pkg):
    """The kernels' division-free quantizer (x times the reciprocal scale,
    the division only within 1e-4 of a rounding boundary) against the
    oracle on quotients exactly at k + 1/2, one ulp either side and at the
    +-127.5 clamp edge (tests/test_quantize_rule.py restates the rule)."""
    from test_quantize_rule import adversarial
    rng = np.random.default_rng(5)
    for amax in (np.float32(3.0e-3), np.float32(0.7), np.float32(17.0), np.float32(2.5e3)):
        x = adversarial(rng, amax)
        x = np.concatenate([x, np.zeros((-x.size) % 4, np.float32)])[None, :]
        q = torch.empty(x.shape, dtype=torch.int8, device="cuda")
        am = torch.empty(1, dtype=torch.float32, device="cuda")
        pkg.shim.check(lib.tl_quantize_int8(dev(x).data_ptr(), 1, x.shape[1], 1, q.data_ptr(), am.data_ptr(),
                                            stream()), "quantize")
        want, _ = G.quantize_int8(x)
        np.testing.assert_array_equal(q.cpu().numpy(), want, err_msg=str(amax))


def test_quantized_linear_matches_reference_fixture(pkg, golden, lib):
    d = golden["quant_cases"]
    for i in range(4):
        out, dbg = pkg.quantized_linear(d[f"l{i}_x"], d[f"l{i}_w"], capture_arrays=True)
        np.testing.assert_array_equal(dbg["accum_int32"], d[f"l{i}_acc"])
        np.testing.assert_array_equal(dbg["input_q"], d[f"l{i}_xq"])
        np.testing.assert_array_equal(out, d[f"l{i}_out"])


@pytest.mark.parametrize("rows,cols", [(3, 64), (7, 256), (5, 2048), (2, 5632), (1, 704)])
def test_rmsnorm_bit_exact(pkg, lib, rows, cols):
    rng = np.random.default_rng(rows * cols)
    x = (rng.standard_normal((rows, cols), dtype=np.float32) * rng.uniform(0.01, 30)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(cols, dtype=np.float32)).astype(np.float32)
    np.testing.assert_array_equal(pkg.rms_norm(x, g, 1e-5), G.rms_norm(x, g, 1e-5))


def test_rmsnorm_reference_fixture(pkg, golden, lib):
    d = golden["small_model"]
    np.testing.assert_array_equal(pkg.rms_norm(d["rms_x"], d["rms_g"], 1e-5), d["rms_out"])


@pytest.mark.parametrize("rows,vocab,hidden", [(1, 32000, 2048), (3, 512, 256), (8, 1000, 2048)])
def test_lmhead_argmax_bit_exact(pkg, lib, rows, vocab, hidden):
    rng = np.random.default_rng(vocab + rows)
    x = rng.standard_normal((rows, hidden), dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(hidden, dtype=np.float32)).astype(np.float32)
    wf = (rng.standard_normal((hidden, vocab), dtype=np.float32) * 0.02).astype(np.float32)
    lw = pkg.quantize_weight(wf, "channel")
    tok = torch.empty(rows, dtype=torch.int32, device="cuda")
    logits = torch.empty((rows, vocab), dtype=torch.float32, device="cuda")
    pkg.shim.check(lib.tl_lmhead_argmax(dev(x).data_ptr(), dev(g).data_ptr(), 1e-5,
                                        dev(np.ascontiguousarray(lw.w.T)).data_ptr(), dev(lw.scale).data_ptr(),
                                        rows, vocab, hidden, tok.data_ptr(), logits.data_ptr(), stream()),
                   "lmhead")
    ref = []
    for r in range(rows):
        h = G.rms_norm(x[r:r + 1], g, 1e-5)
        lg, _, _, _ = G.linear_q(h, lw.w, lw.scale)
        ref.append(lg[0])
    ref = np.array(ref)
    np.testing.assert_array_equal(logits.cpu().numpy(), ref)
    assert list(tok.cpu().numpy()) == [G.argmax_first(r) for r in ref]


def test_argmax_tie_breaks_to_lowest_id(pkg, lib):
    """Equal logits: the lower token id wins (argmax_reduction.sv:47-58)."""
    hidden, vocab = 64, 300
    x = np.ones((1, hidden), np.float32)
    g = np.ones(hidden, np.float32)
    w = np.zeros((hidden, vocab), np.int8)
    w[:, 17] = 5
    w[:, 230] = 5
    w[:, 3] = 4
    s = np.full(vocab, 0.01, np.float64)
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    pkg.shim.check(lib.tl_lmhead_argmax(dev(x).data_ptr(), dev(g).data_ptr(), 1e-5,
                                        dev(np.ascontiguousarray(w.T)).data_ptr(), dev(s).data_ptr(),
                                        1, vocab, hidden, tok.data_ptr(), None, stream()), "lmhead")
    assert int(tok.item()) == 17


def test_invalid_shapes_rejected(pkg, lib):
    a = torch.zeros((1, 24), dtype=torch.int8, device="cuda")
    c = torch.zeros((1, 8), dtype=torch.int32, device="cuda")
    assert lib.tl_gemm_i8(a.data_ptr(), a.data_ptr(), c.data_ptr(), 1, 8, 24, stream()) == 16
    assert lib.tl_gemm_i8(None, a.data_ptr(), c.data_ptr(), 1, 8, 16, stream()) == 16


CONFIG1 = [(m, k, n) for m in (1, 32, 512, 4096) for k in (2048, 5632) for n in (256, 2048, 5632, 32000)]


@pytest.mark.parametrize("m,k,n", CONFIG1)
def test_config1_gemm_sweep_requant(lib, pkg, m, k, n):
    """Benchmark config 1: INT8 x INT8 -> INT32 with per-tensor Q16.16
    requantize to INT8, operands uniform in [-127,127], scale uniform in
    [1e-4, 1e-2]. Bit-exact on 8 sampled rows (all rows for m <= 32)."""
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    w_nk = rng.integers(-127, 128, (n, k), dtype=np.int8)
    scale = rng.uniform(1e-4, 1e-2)
    sq = np.array([C.q16_16_from_float(scale)], dtype=np.uint32)
    out = torch.empty((m, n), dtype=torch.int8, device="cuda")
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    da, dw = dev(a), dev(w_nk)
    pkg.shim.check(lib.tl_gemm_i8_requant(da.data_ptr(), dw.data_ptr(), dev(sq).data_ptr(), 0, 0, out.data_ptr(),
                                          m, n, k, stream()), "requant")
    pkg.shim.check(lib.tl_gemm_i8(da.data_ptr(), dw.data_ptr(), acc.data_ptr(), m, n, k, stream()), "gemm")
    rows = np.arange(m) if m <= 32 else np.sort(rng.choice(m, 8, replace=False))
    ref_acc = G.int8_matmul(a[rows], np.ascontiguousarray(w_nk.T))
    got_acc = acc.cpu().numpy()[rows]
    np.testing.assert_array_equal(got_acc, ref_acc)
    np.testing.assert_array_equal(out.cpu().numpy()[rows], C.requantize_q16(ref_acc, sq[0]))
    assert pkg.shim.load_library().tl_device_error() == 0


@pytest.mark.parametrize("m", [16, 40, 130])
def test_quantized_linear_tc(pkg, lib, m):
    rng = np.random.default_rng(m)
    x = rng.standard_normal((m, 2048), dtype=np.float32)
    w = (rng.standard_normal((2048, 384), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    out, dbg = pkg.quantized_linear(x, w, capture_arrays=True)
    ref, rdbg = G.quantized_linear(x, w)
    np.testing.assert_array_equal(dbg["accum_int32"], rdbg["accum_int32"])
    np.testing.assert_array_equal(out, ref)


def attn_reference(qkv, pos, slot, kc, vc, ks, vs, cos, sin, layer, H, Hkv):
    """NumPy decode attention with the engine's INT8-cache semantics
    (oracle/kv_golden.py): RoPE q/k, append quantized k/v at pos, attend over
    0..pos with dequantized K/V (float64 scores as in the reference)."""
    G = H // Hkv
    out = np.zeros((len(pos), H * 64), np.float32)
    kc, vc = kc.copy(), vc.copy()
    for r, (p, s) in enumerate(zip(pos, slot)):
        row = qkv[r]
        q = row[:H * 64].reshape(H, 1, 64)
        k = row[H * 64:(H + Hkv) * 64].reshape(Hkv, 1, 64)
        v = row[(H + Hkv) * 64:].reshape(Hkv, 1, 64)
        q = G_.rope(q, cos[p:p + 1], sin[p:p + 1])
        k = G_.rope(k, cos[p:p + 1], sin[p:p + 1])
        for h in range(Hkv):
            kc[s, layer, h, p] = G_.quantize_with_scale(k[h, 0], float(ks[s, layer, h]))
            vc[s, layer, h, p] = G_.quantize_with_scale(v[h, 0], float(vs[s, layer, h]))
        kd = kc[s, layer, :, :p + 1].astype(np.float32) * ks[s, layer][:, None, None]
        vd = vc[s, layer, :, :p + 1].astype(np.float32) * vs[s, layer][:, None, None]
        out[r] = G_.attention_core(q, kd, vd, G, np.float64(0.125), False)[0]
    return out, kc, vc


G_ = G


@pytest.mark.parametrize("rows,H,Hkv,positions", [(1, 32, 4, [5]), (1, 32, 4, [300]), (3, 4, 2, [0, 63, 64]),
                                                  (2, 32, 4, [1023, 2047]), (20, 32, 4, list(range(0, 2000, 100)))])
def test_attn_decode_matches_reference(pkg, lib, rows, H, Hkv, positions):
    rng = np.random.default_rng(rows * 31 + H + positions[0])
    L, P = 2, 2048
    slots = rows + 1
    kc = rng.integers(-127, 128, (slots, L, Hkv, P, 64), dtype=np.int8)
    vc = rng.integers(-127, 128, (slots, L, Hkv, P, 64), dtype=np.int8)
    ks = rng.uniform(0.005, 0.03, (slots, L, Hkv)).astype(np.float32)
    vs = rng.uniform(0.005, 0.03, (slots, L, Hkv)).astype(np.float32)
    qkv = rng.standard_normal((rows, (H + 2 * Hkv) * 64), dtype=np.float32)
    pos = np.array(positions, np.int32)
    slot = (np.arange(rows, dtype=np.int32) + 1) % slots
    cos, sin = G.build_rope_cache(P, 64, 10000.0)
    ref, kref, vref = attn_reference(qkv, pos, slot, kc, vc, ks, vs, cos, sin, 1, H, Hkv)
    dkc, dvc = dev(kc), dev(vc)
    out = torch.empty((rows, H * 64), dtype=torch.float32, device="cuda")
    pkg.shim.check(lib.tl_attn_decode(dev(qkv).data_ptr(), dev(pos).data_ptr(), dev(slot).data_ptr(),
                                      dkc.data_ptr(), dvc.data_ptr(), dev(ks).data_ptr(), dev(vs).data_ptr(),
                                      dev(cos).data_ptr(), dev(sin).data_ptr(), 1, L, H, Hkv, P, rows,
                                      out.data_ptr(), stream()), "attn")
    got = out.cpu().numpy()
    err = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
    assert err < 2e-6, err
    np.testing.assert_array_equal(dkc.cpu().numpy(), kref)
    np.testing.assert_array_equal(dvc.cpu().numpy(), vref)


@pytest.mark.parametrize("n_seqs,S,H,Hkv,P", [(1, 1, 32, 4, 2048), (2, 63, 4, 2, 2048), (1, 64, 32, 4, 2048),
                                              (2, 65, 32, 4, 2048), (3, 200, 4, 2, 2048), (1, 2048, 32, 4, 2048),
                                              # cache capacity not a multiple of the 128-key tile
                                              (2, 250, 8, 2, 250)])
def test_attn_prefill_matches_reference(pkg, lib, n_seqs, S, H, Hkv, P):
    """Causal prefill attention over the INT8 cache vs the oracle's attention
    core (float64 scores) on dequantized cache rows."""
    rng = np.random.default_rng(S * 7 + n_seqs + H)
    L, layer, slot_base = 2, 1, 1
    slots = slot_base + n_seqs
    kc = rng.integers(-127, 128, (slots, L, Hkv, P, 64), dtype=np.int8)
    vc = rng.integers(-127, 128, (slots, L, Hkv, P, 64), dtype=np.int8)
    ks = rng.uniform(0.005, 0.03, (slots, L, Hkv)).astype(np.float32)
    vs = rng.uniform(0.005, 0.03, (slots, L, Hkv)).astype(np.float32)
    qkv = (rng.standard_normal((n_seqs * S, (H + 2 * Hkv) * 64)) * 2.0).astype(np.float32)
    ref = np.zeros((n_seqs * S, H * 64), np.float32)
    for i in range(n_seqs):
        sl = slot_base + i
        q = G.split_heads(qkv[i * S:(i + 1) * S, :H * 64], H, 64)
        kd = kc[sl, layer, :, :S].astype(np.float32) * ks[sl, layer][:, None, None]
        vd = vc[sl, layer, :, :S].astype(np.float32) * vs[sl, layer][:, None, None]
        ref[i * S:(i + 1) * S] = G.attention_core(q, kd, vd, H // Hkv, np.float64(0.125), True)
    out = torch.empty((n_seqs * S, H * 64), dtype=torch.float32, device="cuda")
    amax = torch.zeros(n_seqs, dtype=torch.float32, device="cuda")
    pkg.shim.check(lib.tl_attn_prefill(dev(qkv).data_ptr(), S, n_seqs, dev(kc).data_ptr(), dev(vc).data_ptr(),
                                       dev(ks).data_ptr(), dev(vs).data_ptr(), slot_base, layer, L, H, Hkv, P,
                                       out.data_ptr(), amax.data_ptr(), stream()), "attn_prefill")
    got = out.cpu().numpy()
    err = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
    # fp32-level: one warp's fp32 accumulator carries the online softmax over
    # up to 2048 keys (32 rescales); measured 5.9e-6 at S = 2048
    assert err < 1e-5, err
    per_seq = np.abs(got).reshape(n_seqs, -1).max(axis=1)
    np.testing.assert_array_equal(amax.cpu().numpy(), per_seq)
