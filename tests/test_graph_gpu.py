"""CUDA graph capture of the public calls, as a serving loop captures its
decode step: the launches (and their tensor maps, which hold the buffers'
addresses) are recorded once on static buffers, and each replay reads
whatever those buffers hold.  Replays on new inputs written in place must
give bitwise the eager results."""
import pytest
import torch

from tests.conftest import submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")


def fresh_inputs(n, seed, pages):
    w = W.make_uniform(n, pages, seed=seed, device="cuda")
    return w


def test_attention_call_replays_on_new_inputs(dsa):
    n, pages = 64, 256
    w = fresh_inputs(n, 1, pages)
    q_nope, q_pe, idx = w.q_nope.clone(), w.q_pe.clone(), w.sparse_indices.clone()
    out = torch.empty((n, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((n, 16), dtype=torch.float32, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):   # warm-up off the capture (one-time setup, workspace)
        dsa.launch_sparse_attention_c(q_nope, q_pe, w.ckv_cache, w.kpe_cache, idx, w.sm_scale, out, lse)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dsa.launch_sparse_attention_c(q_nope, q_pe, w.ckv_cache, w.kpe_cache, idx, w.sm_scale, out, lse)
    for seed in (2, 3, 4):
        w2 = fresh_inputs(n, seed, pages)
        q_nope.copy_(w2.q_nope)
        q_pe.copy_(w2.q_pe)
        idx.copy_(w2.sparse_indices)
        g.replay()
        torch.cuda.synchronize()
        ro, rl = dsa.kernel(w2.q_nope, w2.q_pe, w.ckv_cache, w.kpe_cache, w2.sparse_indices, w.sm_scale)
        assert torch.equal(out, ro) and torch.equal(lse, rl), f"replay on inputs {seed}"
    assert dsa.check_device_errors() == 0
    del g


def test_small_batch_cluster_merge_replays(dsa):
    """A batch of 3 tokens: the cluster launch (16-CTA clusters) under capture."""
    n, pages = 3, 64
    w = fresh_inputs(n, 11, pages)
    q_nope, q_pe, idx = w.q_nope.clone(), w.q_pe.clone(), w.sparse_indices.clone()
    out = torch.empty((n, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((n, 16), dtype=torch.float32, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        dsa.launch_sparse_attention_c(q_nope, q_pe, w.ckv_cache, w.kpe_cache, idx, w.sm_scale, out, lse)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dsa.launch_sparse_attention_c(q_nope, q_pe, w.ckv_cache, w.kpe_cache, idx, w.sm_scale, out, lse)
    for seed in (12, 13):
        w2 = fresh_inputs(n, seed, pages)
        q_nope.copy_(w2.q_nope)
        q_pe.copy_(w2.q_pe)
        idx.copy_(w2.sparse_indices)
        g.replay()
        torch.cuda.synchronize()
        ro, rl = dsa.kernel(w2.q_nope, w2.q_pe, w.ckv_cache, w.kpe_cache, w2.sparse_indices, w.sm_scale)
        assert torch.equal(out, ro) and torch.equal(lse, rl)
    assert dsa.check_device_errors() == 0
    del g


def test_decode_step_indexer_then_attention_replays(dsa):
    """The indexer's top-k feeding the attention, captured as one graph (the
    score split plan is read from the workspace at run time, so replays keep
    calibrating)."""
    rows = 16
    wi = W.indexer_decode(batch=rows, seq_len=8192, device="cuda")
    pages = wi.k_index_cache.shape[0]
    wa = W.make_uniform(rows, pages, seed=21, device="cuda")
    q_idx, weights = wi.q_index_fp8.clone(), wi.weights.clone()
    topk = torch.empty((rows, 2048), dtype=torch.int32, device="cuda")
    out = torch.empty((rows, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((rows, 16), dtype=torch.float32, device="cuda")

    def step():
        dsa.launch_topk_c(q_idx, wi.k_index_cache, weights, wi.seq_lens, wi.block_table, topk)
        dsa.launch_sparse_attention_c(wa.q_nope, wa.q_pe, wa.ckv_cache, wa.kpe_cache, topk, wa.sm_scale, out, lse)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for seed in (31, 32, 33, 34):
        w2 = W.indexer_decode(seed=seed, batch=rows, seq_len=8192, device="cuda")
        q_idx.copy_(w2.q_index_fp8)
        weights.copy_(w2.weights)
        g.replay()
        torch.cuda.synchronize()
        ref_idx = dsa.topk_indexer(w2.q_index_fp8, wi.k_index_cache, w2.weights, wi.seq_lens, wi.block_table)
        assert torch.equal(topk, ref_idx), f"top-k, replay on inputs {seed}"
        ro, rl = dsa.kernel(wa.q_nope, wa.q_pe, wa.ckv_cache, wa.kpe_cache, ref_idx, wa.sm_scale)
        assert torch.equal(out, ro) and torch.equal(lse, rl), f"attention, replay on inputs {seed}"
    assert dsa.check_device_errors() == 0
    assert dsa.indexer.check_errors() == 0
    del g
