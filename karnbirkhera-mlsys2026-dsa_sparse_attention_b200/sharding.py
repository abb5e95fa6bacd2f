"""Batch-row sharding of query tokens across the GPUs of one node.

Query tokens are independent, so the path shards with no collective on the
hot path: rank r of W takes a contiguous range of batch rows (whole
sequences), holds only those sequences' KV pages in its own pool, and runs the
single-GPU operator on them.  Outputs stay sharded; the benchmark only reduces
its timing (max over ranks) outside the timed region.
"""
from __future__ import annotations

from . import workloads


def row_range(num_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous near-equal split of [0, num_rows) into `world` parts."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    return (rank * num_rows) // world, ((rank + 1) * num_rows) // world


def shard_config5(world: int, rank: int, seed: int = 5, device="cpu",
                  num_seqs: int = workloads.CFG5_SEQS,
                  seq_tokens: int = workloads.CFG5_SEQ_TOKENS) -> workloads.Workload:
    """This rank's part of benchmark config 5: whole sequences, their pages
    only, indices remapped to the local pool."""
    a, b = row_range(num_seqs, world, rank)
    return workloads.config5(seed=seed, device=device, seq_begin=a, seq_end=b, seq_tokens=seq_tokens)


def shard_config2(world: int, rank: int, seed: int = 2, device="cpu", **kw) -> workloads.Workload:
    """Weak scaling of config 2: every rank serves its own 64-token decode
    batch (its own sequences and pool); the job's batch is 64 * world tokens."""
    return workloads.config2(seed=seed + 1009 * rank, device=device, **kw)
