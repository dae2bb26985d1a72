"""Tensor-parallel prefill on 2 GPUs (tl_tp_create_ex, both exchanges): logits and the rank's
INT8 KV-cache bytes must be bit-identical to the single-GPU engine on the
same weights -- a small model from the oracle's archive (loaded through the
full host view, sliced by the engine) and TinyLlama-size random weights
(each rank draws its slice of the single-GPU model). Skipped below 2 GPUs."""

from __future__ import annotations

import multiprocessing as mp

import numpy as np
import pytest

from dist_workers import gpu_tp_prefill_rank

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("exchange", ["allreduce", "allgather"])
def test_tp2_prefill_bit_identical_to_one_gpu(pkg, exchange):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ids = (pkg.tp_unique_id(), pkg.tp_unique_id())
    prompt = [int(t) for t in np.random.default_rng(10).integers(0, 512, 23)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=gpu_tp_prefill_rank, args=(r, world, ids, prompt, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=600) for _ in range(world))
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
    finally:  # a rank left waiting in a collective must not outlive the test
        for p in procs:
            if p.is_alive():
                p.terminate()
    r0 = res[0]
    for rank in range(world):
        np.testing.assert_array_equal(res[rank]["small_logits"], r0["one_small_logits"])
        np.testing.assert_array_equal(res[rank]["big_logits"], r0["one_big_logits"])
        hs = res[rank]["small_k"].shape[0]
        np.testing.assert_array_equal(res[rank]["small_k"], r0["one_small_k"][rank * hs:(rank + 1) * hs])
        hb = res[rank]["big_k"].shape[0]
        np.testing.assert_array_equal(res[rank]["big_k"], r0["one_big_k"][rank * hb:(rank + 1) * hb])
