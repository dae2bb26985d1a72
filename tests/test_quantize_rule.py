"""The kernels' division-free INT8 quantizer (quantize_one_inv in
csrc/common.cuh) restated in NumPy float32 and checked against the
reference rule of model/tinyllama_gemm_int8.py:36-42 (oracle
golden.quantize_int8): a = x * fl(1 / scale), rint(a) unless a lies within
1e-4 of a half-integer (then rint(x / scale)), |a| >= 128 clamps. Inputs
include quotients exactly at k + 1/2, one float32 ulp either side of them,
the +-127.5 clamp edge and random values, over scales from 1e-6 to 1e4."""

import numpy as np

from oracle import golden as G

f32 = np.float32


def device_rule(x, scale):
    s = f32(scale)
    inv = f32(1) / s
    a = (x * inv).astype(f32)
    q = np.rint(a)
    near = np.abs(a - q) > f32(0.4999)
    q = np.where(near, np.rint((x / s).astype(f32)), q)
    q = np.where(np.abs(a) >= 128, np.sign(a) * 127, q)
    return np.clip(q, -127, 127).astype(np.int8)


def adversarial(rng, amax):
    s = f32(np.float64(amax) / 127.0)
    k = np.arange(-128, 128, dtype=f32)
    half = ((k + f32(0.5)) * s).astype(f32)
    cases = [half, np.nextafter(half, f32(np.inf)), np.nextafter(half, f32(-np.inf)),
             (rng.uniform(-1, 1, 4096) * amax).astype(f32)]
    x = np.concatenate(cases)
    x = x[np.abs(x) <= f32(amax)]  # the tensor's own absmax stays amax
    return np.concatenate([x, np.array([amax, -amax, 0.0], f32)])


def test_division_free_rule_matches_reference():
    rng = np.random.default_rng(11)
    total = 0
    for amax in np.exp(rng.uniform(np.log(1e-4), np.log(1e6), 60)).astype(f32):
        x = adversarial(rng, amax)
        want, scale = G.quantize_int8(x)
        np.testing.assert_array_equal(device_rule(x, scale), want, err_msg=f"amax {amax}")
        total += x.size
    assert total > 60 * 4000
