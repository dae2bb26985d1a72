"""Data-parallel decode plumbing (bench.py --gpus N) on CPU ranks over gloo.

Batched decode shards by sequence with no collective on the data path; these
tests cover the host side: sequence partition, per-rank work, barrier and the
max-over-ranks timing reduction, with world_size 2."""

from __future__ import annotations

import multiprocessing as mp
import socket

import pytest

from dist_workers import decode_shard_rank
from helpers import small_model
from oracle.kv_golden import KVGolden


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_covers_exactly_once(pkg):
    rp = pkg.replicas
    for n in (0, 1, 7, 64, 65, 130):
        for world in (1, 2, 3, 4, 8):
            blocks = [rp.partition(n, world, r) for r in range(world)]
            seen = [i for first, count in blocks for i in range(first, first + count)]
            assert seen == list(range(n))
            counts = [c for _, c in blocks]
            assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        rp.partition(4, 2, 2)
    assert rp.aggregate_rate([100, 100], [10.0, 20.0]) == pytest.approx(200 / 0.02)


def test_two_rank_decode_shards_match_single_process():
    world, n_global, max_new = 2, 5, 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=decode_shard_rank, args=(r, world, port, n_global, max_new, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    merged = {}
    for rank, first, count, toks, t_max, n_tok, rate in results:
        assert t_max == 20.0                      # slowest rank's time
        assert n_tok == n_global * max_new        # every sequence decoded once
        assert rate == pytest.approx(n_global * max_new / 0.020)
        merged.update(toks)
    assert sorted(merged) == list(range(n_global))
    # the sharded run equals one process decoding every sequence
    import numpy as np
    prompts = np.random.default_rng(123).integers(0, 512, (n_global, 5))
    qm = small_model(seed=3, layers=1)
    for i in range(n_global):
        assert merged[i] == KVGolden(qm).generate(prompts[i].tolist(), max_new, eos_id=0xFFFFFFFF)[0]
