"""Multi-GPU plumbing for batched decode: one process per GPU, independent
sequences, no collective on the data path.

Batched decode (the reference's run_generate loop, model/tinyllama_gemm_int8.py:629-685,
run once per sequence) shards by sequence: every rank holds a full weight
replica and the KV cache of its own sequences only, and no rank ever needs
another rank's activations. The only cross-rank traffic is host-side
bookkeeping: a barrier around the timed region and the max of the ranks'
device times (the job is as slow as its slowest rank). torch.distributed
carries it, over NCCL on GPUs and gloo on CPU (which is how it is tested).
"""

from __future__ import annotations

import datetime
import os


def env_rank() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def partition(n_global: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block of sequences owned by ``rank``: (first, count).

    The first ``n_global % world`` ranks take one extra sequence, so blocks
    differ by at most one and cover [0, n_global) exactly once."""
    if world <= 0 or not 0 <= rank < world or n_global < 0:
        raise ValueError(f"bad partition request: n={n_global} world={world} rank={rank}")
    base, extra = divmod(n_global, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def rank_seed(base: int, rank: int) -> int:
    """Seed of a rank's synthetic prompts: distinct sequences on every rank."""
    return base + rank


class Group:
    """The process group used for the step barrier and timing reductions.

    ``world == 1`` needs no process group; every method then acts locally."""

    def __init__(self, world: int, backend: str = "nccl", device=None, timeout_s: float = 300.0):
        self.world = world
        self.dist = None
        self.device = device
        if world > 1:
            import torch.distributed as dist
            kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
            if backend == "nccl" and device is not None:
                kw["device_id"] = device
            dist.init_process_group(backend, **kw)
            self.dist = dist

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def _reduce(self, value: float, op_name: str) -> float:
        if not self.dist:
            return float(value)
        import torch
        dev = self.device if self.device is not None else "cpu"
        t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
        self.dist.all_reduce(t, op=getattr(self.dist.ReduceOp, op_name))
        return float(t.item())

    def max(self, value: float) -> float:
        """Max over ranks (timings: the job ends with its slowest rank)."""
        return self._reduce(value, "MAX")

    def sum(self, value: float) -> float:
        """Sum over ranks (work counts)."""
        return self._reduce(value, "SUM")

    def close(self):
        if self.dist:
            self.dist.destroy_process_group()
            self.dist = None


def aggregate_rate(units_per_rank: list[float] | float, ms_per_rank: list[float] | float,
                   group: Group | None = None) -> float:
    """Whole-job rate: units processed by all ranks / the slowest rank's time.

    With a group, each rank passes its own scalars and the reduction runs
    over the group; without one, lists of every rank's values are given."""
    if group is not None:
        return group.sum(units_per_rank) / (group.max(ms_per_rank) / 1e3)
    return float(sum(units_per_rank)) / (max(ms_per_rank) / 1e3)
