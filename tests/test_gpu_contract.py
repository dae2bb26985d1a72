"""Contract-mode operators (GPU): the hardware's Q16.16 wrapper chain
(tl_contract_rmsnorm / silu / softmax / rope, tl_residual_add_i32) against
the reference exporter's own cases (tests/golden/contract_mode.npz and the
RoPE cases of contract.npz, written by model/export_fpga_vectors.py) and,
at larger sizes, against oracle/contract.py (pinned to the same cases on
CPU).

Exact: RMSNorm (no transcendental; NumPy's summation order), RoPE, the
residual add (including sums that wrap modulo 2^32). SiLU and softmax call
the device expf where the reference calls NumPy's exp, which can differ in
the last float32 bit: their Q16.16 outputs are within 1 unit of the
reference's and their INT8 outputs within 1 LSB, on a small fraction of
elements (bounded below)."""

import numpy as np
import pytest

from oracle import contract as K

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def near(got, want, frac):
    d = np.abs(np.asarray(got, np.int64) - np.asarray(want, np.int64))
    assert d.max() <= 1 and np.mean(d != 0) <= frac, (int(d.max()), float(np.mean(d != 0)))


def test_rmsnorm_exact(pkg, golden):
    d = golden["contract_mode"]
    for m in ("prefill", "decode"):
        y16, yq = pkg.contract_rmsnorm(d[f"rms_{m}_x_q"], d[f"rms_{m}_in_q16"], d[f"rms_{m}_gamma_q16"],
                                       float(d["rms_eps"]), d[f"rms_{m}_out_q16"])
        np.testing.assert_array_equal(y16, d[f"rms_{m}_y_q16"])
        np.testing.assert_array_equal(yq, d[f"rms_{m}_y_q"])
    rng = np.random.default_rng(1)
    x = rng.integers(-127, 128, (64, 2048)).astype(np.int8)
    g = rng.integers(50000, 80000, 2048).astype(np.int32)
    y16, yq = pkg.contract_rmsnorm(x, 1234, g, 1e-5, 900)
    w16, wq, _ = K.rmsnorm_contract(x, 1234, g, 1e-5, 900)
    np.testing.assert_array_equal(y16, w16)
    np.testing.assert_array_equal(yq, wq)


def test_silu(pkg, golden):
    d = golden["contract_mode"]
    for m in ("prefill", "decode"):
        y16, yq = pkg.contract_silu(d[f"silu_{m}_x_q"], d[f"silu_{m}_in_q16"], d[f"silu_{m}_out_q16"])
        near(y16, d[f"silu_{m}_y_q16"], 0.05)
        near(yq, d[f"silu_{m}_y_q"], 0.02)
    x = np.random.default_rng(2).integers(-127, 128, 200000).astype(np.int8)
    y16, yq = pkg.contract_silu(x, 3100, 2500)
    w16, wq, _ = K.silu_contract(x, 3100, 2500)
    near(y16, w16, 0.05)
    near(yq, wq, 0.01)


def test_softmax_probability_scale(pkg, golden):
    d = golden["contract_mode"]
    for m in ("prefill", "decode"):
        n = int(d[f"sm_{m}_rows"])
        p16, pq = pkg.contract_softmax(d[f"sm_{m}_score"][:n], d[f"sm_{m}_scale_q16"])
        near(p16, d[f"sm_{m}_prob_q16"][:n], 0.05)
        near(pq, d[f"sm_{m}_prob_q"][:n], 0.02)
    rng = np.random.default_rng(3)
    for cols in (5, 64, 100, 128):
        sc = rng.integers(-200000, 200000, (97, cols)).astype(np.int32)
        sc[::7, cols // 2:] = -1000000000  # masked keys, as the exporter's tiles
        p16, pq = pkg.contract_softmax(sc, 3)
        w16, wq, _ = K.softmax_contract(sc, 3)
        near(p16, w16, 0.05)
        near(pq, wq, 0.02)
        assert pq.min() >= 0 and pq.max() <= 127


def test_rope_int8_exact(pkg, golden):
    c = golden["contract"]
    for key in ("rope_q", "rope_k"):
        got = pkg.contract_rope(c[key], c["rope_cos_q16"], c["rope_sin_q16"])
        np.testing.assert_array_equal(got, c[f"{key}_out"])
    rng = np.random.default_rng(4)
    x = rng.integers(-127, 128, (4096, 64)).astype(np.int8)
    cs = rng.integers(-65536, 65537, (4096, 64)).astype(np.int32)
    sn = rng.integers(-65536, 65537, (4096, 64)).astype(np.int32)
    np.testing.assert_array_equal(pkg.contract_rope(x, cs, sn), K.rope_int8(x, cs, sn))


def test_residual_add_wraps(pkg, golden):
    d = golden["contract_mode"]
    np.testing.assert_array_equal(pkg.residual_add_i32(d["res_a"], d["res_b"]), d["res_sum"])
    a = np.array([2**31 - 5, -2**31 + 3, 7], np.int64).astype(np.int32)
    b = np.array([10, -10, -9], np.int32)
    np.testing.assert_array_equal(pkg.residual_add_i32(a, b), K.residual_add_i32(a, b))


def test_rejects_bad_shapes(pkg):
    with pytest.raises(pkg.TLError):
        pkg.contract_softmax(np.zeros((2, 129), np.int32), 1)
