"""The device-timeout path of the attention kernel.

Every pipeline wait of the kernel is bounded; a wait that reaches its limit
makes the CTA stop, drain its own copies and tensor-core operations (under a
separate bound of at least 2 s, so nothing is still in flight when the CTA
frees its tensor memory and exits) and raise DSA_DEVICE_ERR_TIMEOUT in the
workspace's error word.  The reference's waits have no bound at all
(solution/cuda/kernel.cu:105-116).

The wait is made to run out with the library's test hook
(dsa_sparse_attention_test_hold): every CTA first waits for a workspace word
that nothing sets, under a pipeline limit of 1 ms
(dsa_sparse_attention_set_wait_timeout_ns).  Nothing faults and nothing is
left running: the waiting role gives up, the others see the abort, drain and
exit.  The call must report DSA_ERR_DEVICE_TIMEOUT, and the next call with
the default limit, on the same workspace, must be correct.
"""
import pytest
import torch

from oracle.dsa_oracle import compact_pool, sparse_attention_oracle
from tests.conftest import assert_lse_close, assert_output_close, pkg, submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _oracle(w, tokens):
    ckv, kpe, idx_c = compact_pool(w.ckv_cache, w.kpe_cache, w.sparse_indices[tokens])
    return sparse_attention_oracle(w.q_nope[tokens].cpu(), w.q_pe[tokens].cpu(), ckv.cpu(), kpe.cpu(),
                                   idx_c.cpu(), w.sm_scale)


@pytest.mark.parametrize("num_tokens", [4, 64])
def test_wait_timeout_is_reported_and_the_next_call_is_clean(num_tokens):
    dsa = pkg()
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    W = submodule("workloads")
    w = W.config2(device="cuda", num_tokens=num_tokens, pool_pages=4096)
    out = torch.empty((num_tokens, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((num_tokens, 16), dtype=torch.float32, device="cuda")
    dsa.launch_sparse_attention_c(*w.args(), out, lse)
    torch.cuda.synchronize()
    assert dsa.check_device_errors() == 0
    try:
        assert lib.dsa_sparse_attention_set_wait_timeout_ns(1_000_000) == lib_mod.DSA_OK
        assert lib.dsa_sparse_attention_test_hold(1) == lib_mod.DSA_OK
        dsa.launch_sparse_attention_c(*w.args(), out, lse)
        torch.cuda.synchronize()
    finally:
        assert lib.dsa_sparse_attention_test_hold(0) == lib_mod.DSA_OK
        assert lib.dsa_sparse_attention_set_wait_timeout_ns(0) == lib_mod.DSA_OK
    with pytest.raises(lib_mod.DsaError) as err:
        dsa.check_device_errors()   # reads and clears the error word and the merge state
    assert err.value.status == lib_mod.DSA_ERR_DEVICE_TIMEOUT
    # the context and the workspace are usable: a normal call is correct
    out2, lse2 = dsa.kernel(*w.args())
    torch.cuda.synchronize()
    assert dsa.check_device_errors() == 0
    tokens = list(range(min(num_tokens, 8)))
    o_ref, l_ref = _oracle(w, tokens)
    assert_output_close(out2[tokens], o_ref)
    assert_lse_close(lse2[tokens], l_ref)
