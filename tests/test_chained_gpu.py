"""Kernels chained on one stream without host synchronisation.

Every library kernel is launched with programmatic stream serialization: its
grid may be scheduled while the previous kernel on the stream is finishing and
waits (griddepcontrol.wait) before it reads anything.  These tests run calls
back to back, with no synchronisation between them, and require exactly the
results of the same calls made one at a time: consecutive attention calls of
different sizes (the split plan and the workspace's ticket counters change
from call to call), and the indexer followed by the attention on its top-k
slot ids (one DSA sparse attention layer).
"""
import pytest
import torch

from tests.conftest import submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")


def test_attention_calls_back_to_back(dsa):
    """Token counts 64, 5, 128, 1, 64, 33: each call's output equals the same
    call made in isolation, bitwise."""
    works = [W.make_uniform(n, 96, seed=40 + i, device="cuda") for i, n in enumerate((64, 5, 128, 1, 64, 33))]
    alone = []
    for w in works:
        alone.append(dsa.kernel(*w.args()))
        torch.cuda.synchronize()
    outs = [(torch.empty_like(o), torch.empty_like(l)) for o, l in alone]
    for _ in range(2):
        for w, (o, l) in zip(works, outs):
            dsa.launch_sparse_attention_c(*w.args(), o, l)
    torch.cuda.synchronize()
    assert dsa.check_device_errors() == 0
    for (o, l), (ro, rl) in zip(outs, alone):
        assert torch.equal(o, ro) and torch.equal(l, rl)


def test_indexer_then_attention(dsa):
    """launch_topk_c then launch_sparse_attention_c on its output, twice over
    two workloads, no synchronisation: the same slot ids and attention output
    as the calls made one at a time."""
    cases = []
    for seed in (51, 52):
        wi = W.indexer_small(seed=seed, device="cuda")
        pool = wi.k_index_cache.shape[0]
        wa = W.make_uniform(wi.batch, pool, seed=seed + 100, device="cuda")
        cases.append((wi, wa))
    alone = []
    for wi, wa in cases:
        ids = dsa.topk_indexer(*wi.args())
        torch.cuda.synchronize()
        o, l = dsa.kernel(wa.q_nope, wa.q_pe, wa.ckv_cache, wa.kpe_cache, ids, wa.sm_scale)
        torch.cuda.synchronize()
        alone.append((ids, o, l))
    got = []
    for wi, wa in cases:
        ids = torch.empty((wi.batch, 2048), dtype=torch.int32, device="cuda")
        o = torch.empty((wi.batch, 16, 512), dtype=torch.bfloat16, device="cuda")
        l = torch.empty((wi.batch, 16), dtype=torch.float32, device="cuda")
        got.append((ids, o, l))
    for _ in range(2):
        for (wi, wa), (ids, o, l) in zip(cases, got):
            dsa.launch_topk_c(*wi.args(), ids)
            dsa.launch_sparse_attention_c(wa.q_nope, wa.q_pe, wa.ckv_cache, wa.kpe_cache, ids, wa.sm_scale, o, l)
    torch.cuda.synchronize()
    assert dsa.check_device_errors() == 0
    assert dsa.indexer.check_errors() == 0
    for (ids, o, l), (rids, ro, rl) in zip(got, alone):
        assert torch.equal(ids, rids)
        assert torch.equal(o, ro) and torch.equal(l, rl)
