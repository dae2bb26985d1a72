"""Tensor-parallel prefill decomposition on CPU ranks over gloo (world 2).

The engine's TP-2/4 prefill (tl_tp_create_ex) splits by KV head, combines
the activation maxima before the O and down input quantization with an
all-reduce max, and either all-reduces the INT32 partial sums of row-split O
and down (``allreduce``) or all-gathers their INT8 inputs (``allgather``).
Restated over the oracle's blocks, every rank's logits and its kv heads'
INT8 cache bytes must equal the single-process oracle's bit for bit, with
either exchange."""

from __future__ import annotations

import multiprocessing as mp
import socket

import numpy as np
import pytest

from dist_workers import tp_prefill_rank
from helpers import small_model
from oracle.kv_golden import KVGolden


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("exchange", ["allreduce", "allgather"])
def test_tp2_prefill_equals_single_process(exchange):
    world, seed = 2, 9
    prompt = [int(t) for t in np.random.default_rng(10).integers(0, 512, 23)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=tp_prefill_rank, args=(r, world, port, seed, prompt, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ora = KVGolden(small_model(seed=seed, layers=2, granularity="channel"), kv="int8")
    ref = ora.prefill(prompt)
    hr = ora.cfg["num_key_value_heads"] // world
    for rank, logits, k_local in res:
        np.testing.assert_array_equal(logits, ref)
        np.testing.assert_array_equal(k_local, ora.k_cache[:, rank * hr:(rank + 1) * hr, :len(prompt)])
