"""Small parity cases shared by the golden-fixture generator and the tests.

Every case is rebuilt from a seeded generator; the fixtures hold checksums of
the inputs the reference saw, so a changed generator is caught, not silently
compared against stale outputs.
"""
from __future__ import annotations

import importlib

import torch

W = importlib.import_module("karnbirkhera-mlsys2026-dsa_sparse_attention_b200.workloads")

INPUT_KEYS = ("q_nope", "q_pe", "ckv_cache", "kpe_cache", "sparse_indices")


def checksum(t: torch.Tensor) -> int:
    """Order-sensitive 64-bit checksum of a tensor's bytes."""
    b = t.detach().cpu().contiguous().view(-1).view(torch.uint8).to(torch.int64)
    w = torch.arange(1, b.numel() + 1, dtype=torch.int64) % 1000003
    return int((b * w).sum().item())


def n1_p1():
    """One token, one page: 64 valid slots then 1984 x -1."""
    return W.make_uniform(1, 1, seed=11)


def n3_p40():
    """Full 2048-wide rows over a 40-page pool."""
    return W.make_uniform(3, 40, seed=12)


def empty_and_single():
    """Token 0 all padding (-> output 0, lse -inf); token 1 a single valid index."""
    w = W.make_uniform(2, 40, seed=13)
    w.sparse_indices[0, :] = -1
    w.sparse_indices[1, 1:] = -1
    return w


def dup_and_holes():
    """Token 0 repeats its first 1024 slots; token 1 has every third slot padded."""
    w = W.make_uniform(2, 40, seed=14)
    w.sparse_indices[0, 1024:] = w.sparse_indices[0, :1024].clone()
    w.sparse_indices[1, ::3] = -1
    return w


def config1():
    """Benchmark config 1 (4 tokens, 128 pages)."""
    return W.config1()


CASES = {"n1_p1": n1_p1, "n3_p40": n3_p40, "empty_and_single": empty_and_single,
         "dup_and_holes": dup_and_holes, "config1": config1}
