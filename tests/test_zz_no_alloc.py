"""The allocation-free entry point, dsa_sparse_attention_fwd_noalloc.

It exists for callers that cannot allocate device memory (a serving process
whose whole GPU memory is a fixed arena handed out at start-up, a plugin host
that forbids cudaMalloc), so it keeps its scratch in a fixed device array
inside the library.  Here it is called through the C ABI, twice in a row with
different batches, and each result is checked against the workspace-based
entry point with the suite's tolerances.  The file name sorts last so that a
run that stops at the first failure has already run every other test; the
test needs no state from them and passes on its own in a fresh process.
"""
import pytest
import torch

from tests.conftest import assert_lse_close, assert_output_close, pkg, submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _noalloc(lib, w, out, lse):
    return lib.dsa_sparse_attention_fwd_noalloc(
        w.q_nope.data_ptr(), w.q_pe.data_ptr(), w.ckv_cache.data_ptr(), w.kpe_cache.data_ptr(),
        w.sparse_indices.data_ptr(), w.num_tokens, w.num_pages, w.sm_scale, out.data_ptr(), lse.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    dsa = pkg()
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    W = submodule("workloads")
    # two different batches back to back: a plan where every token spans many
    # CTAs, then one where CTAs span several tokens (both go through the merge)
    batches = [W.make_uniform(5, 64, seed=31, device="cuda", pad=300),
               W.config2(device="cuda", num_tokens=200, pool_pages=4096)]
    for w in batches:
        ref_out, ref_lse = dsa.kernel(*w.args())
        out = torch.full_like(ref_out, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        st = _noalloc(lib, w, out, lse)
        assert st == lib_mod.DSA_OK, lib_mod.status_string(st)
        torch.cuda.synchronize()
        assert_output_close(out, ref_out)
        assert_lse_close(lse, ref_lse)


def test_noalloc_rejects_bad_arguments_without_device_work():
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    assert lib.dsa_sparse_attention_fwd_noalloc(None, None, None, None, None, -1, 1, 0.1, None, None, None) \
        == lib_mod.DSA_ERR_INVALID_ARGUMENT
    assert lib.dsa_sparse_attention_fwd_noalloc(None, None, None, None, None, 0, 1, 0.1, None, None, None) \
        == lib_mod.DSA_OK
