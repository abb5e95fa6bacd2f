"""Small batches merged inside thread-block clusters.

With one 128-slot block per CTA and every token's 16 CTAs resident as one
cluster (up to 7 tokens on a B200), the library merges each token through
distributed shared memory instead of through the workspace records.  The
combine is the same (segments in block order, the same reductions), so the
two merges must agree bit for bit; both are also checked against the CPU
oracle.  dsa_sparse_attention_set_cluster_merge(0) selects the workspace
merge for the comparison run.
"""
import pytest
import torch

from oracle.dsa_oracle import compact_pool, sparse_attention_oracle
from tests.conftest import assert_lse_close, assert_output_close, pkg, submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _oracle(w):
    ckv, kpe, idx_c = compact_pool(w.ckv_cache, w.kpe_cache, w.sparse_indices)
    return sparse_attention_oracle(w.q_nope.cpu(), w.q_pe.cpu(), ckv.cpu(), kpe.cpu(), idx_c.cpu(), w.sm_scale)


@pytest.mark.parametrize("num_tokens,pad", [(1, 0), (3, 517), (6, 0), (7, 1800)])
def test_cluster_merge_is_bitwise_the_workspace_merge(num_tokens, pad):
    dsa = pkg()
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    W = submodule("workloads")
    # pad = 1800: most blocks of a token are empty (segments with no key)
    w = W.make_uniform(num_tokens, 256, seed=700 + num_tokens, device="cuda", pad=pad)
    results = []
    try:
        for enable in (0, 1):
            assert lib.dsa_sparse_attention_set_cluster_merge(enable) == lib_mod.DSA_OK
            out, lse = dsa.kernel(*w.args())
            dsa.check_device_errors()
            results.append((out.clone(), lse.clone()))
    finally:
        lib.dsa_sparse_attention_set_cluster_merge(1)
    (o_ws, l_ws), (o_cl, l_cl) = results
    assert torch.equal(o_cl, o_ws), "cluster merge output differs from the workspace merge"
    assert torch.equal(l_cl, l_ws), "cluster merge lse differs from the workspace merge"
    o_ref, l_ref = _oracle(w)
    assert_output_close(o_cl, o_ref)
    assert_lse_close(l_cl, l_ref)


def test_cluster_merge_back_to_back_calls_of_different_sizes():
    """Cluster launches (1..7 tokens) and workspace launches (8, 40 tokens)
    queued on one stream without synchronisation, each checked against the
    oracle afterwards."""
    dsa = pkg()
    W = submodule("workloads")
    cases = [W.make_uniform(n, 256, seed=900 + n, device="cuda") for n in (2, 8, 7, 40, 1)]
    outs = [dsa.kernel(*w.args()) for w in cases]
    dsa.check_device_errors()
    for w, (o, l) in zip(cases, outs):
        o_ref, l_ref = _oracle(w)
        assert_output_close(o, o_ref)
        assert_lse_close(l, l_ref)
