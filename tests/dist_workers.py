"""Rank bodies for the multi-process CPU tests (gloo). Spawned children import
this module by name, so it holds no pytest state."""

from __future__ import annotations

import os

import numpy as np


def _package():
    from conftest import load_package
    return load_package()


def decode_shard_rank(rank: int, world: int, port: int, n_global: int, max_new: int, out_q):
    """One data-parallel decode rank: greedy-decode the sequences this rank
    owns with the KV-cached oracle, then take part in the step bookkeeping
    (barrier, max-over-ranks time, sum of token counts). Nothing crosses
    ranks on the data path."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from helpers import small_model
    from oracle.kv_golden import KVGolden
    rp = _package().replicas
    r, w, lr = rp.env_rank()
    assert (r, w, lr) == (rank, world, rank)
    group = rp.Group(w, backend="gloo", timeout_s=60)
    try:
        first, count = rp.partition(n_global, w, r)
        prompts = np.random.default_rng(123).integers(0, 512, (n_global, 5))
        qm = small_model(seed=3, layers=1)
        toks = {}
        for i in range(first, first + count):
            toks[i] = KVGolden(qm).generate(prompts[i].tolist(), max_new, eos_id=0xFFFFFFFF)[0]
        group.barrier()
        fake_ms = 10.0 * (r + 1)  # distinct per rank: the reduction must pick the slowest
        t_max = group.max(fake_ms)
        n_tok = group.sum(sum(len(t) for t in toks.values()))
        rate = rp.aggregate_rate(sum(len(t) for t in toks.values()), fake_ms, group)
        out_q.put((rank, first, count, toks, t_max, n_tok, rate))
    finally:
        group.close()
