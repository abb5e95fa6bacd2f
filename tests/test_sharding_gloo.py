"""Batch-row sharding across 2 ranks (gloo, CPU): each rank builds only its
sequences' pool, runs the oracle on its shard, and the gathered outputs equal
the unsharded run bit for bit.  Exercises the multi-GPU host logic without a GPU."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

NSEQ = 4
SEQ_TOKENS = 4096


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle.dsa_oracle import sparse_attention_oracle
    from tests.conftest import submodule
    sh = submodule("sharding")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = sh.shard_config5(world, rank, num_seqs=NSEQ, seq_tokens=SEQ_TOKENS)
        out, lse = sparse_attention_oracle(*w.args())
        outs = [torch.empty((NSEQ * 4 // world, 16, 512), dtype=torch.float32) for _ in range(world)]
        lses = [torch.empty((NSEQ * 4 // world, 16), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(outs, out.float())
        dist.all_gather(lses, lse)
        # the timing reduction the benchmark uses: max over ranks
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            torch.save({"out": torch.cat(outs), "lse": torch.cat(lses), "tmax": t.item()},
                       os.path.join(result_dir, "gathered.pt"))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_matches_unsharded(tmp_path):
    from oracle.dsa_oracle import sparse_attention_oracle
    from tests.conftest import submodule
    W = submodule("workloads")
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    got = torch.load(tmp_path / "gathered.pt")
    full = W.config5(seq_begin=0, seq_end=NSEQ, seq_tokens=SEQ_TOKENS)
    out, lse = sparse_attention_oracle(*full.args())
    assert torch.equal(got["out"], out.float())
    assert torch.equal(got["lse"], lse)
    assert got["tmax"] == 2.0
