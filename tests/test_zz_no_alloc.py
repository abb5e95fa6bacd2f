"""The allocation-free entry point, dsa_sparse_attention_fwd_noalloc.

It exists for callers that cannot allocate device memory (a serving process
whose whole GPU memory is a fixed arena handed out at start-up, a plugin host
that forbids cudaMalloc), so it keeps its scratch in a fixed device array
inside the library.  Here it is called through the C ABI three times in a row:
a batch, a larger batch with another plan, then the first batch again, so
that records and counters the larger call leaves in the shared array must not
leak into the next result.  Each result must be bitwise the workspace-based
entry point's (same kernel, same plan), and is also checked against the CPU
oracle with the suite's tolerances.  The file name sorts last so that a run
that stops at the first failure has already run every other test; the test
needs no state from them and passes on its own in a fresh process.
"""
import pytest
import torch

from oracle.dsa_oracle import compact_pool, sparse_attention_oracle
from tests.conftest import assert_lse_close, assert_output_close, pkg, submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _noalloc(lib, w, out, lse):
    return lib.dsa_sparse_attention_fwd_noalloc(
        w.q_nope.data_ptr(), w.q_pe.data_ptr(), w.ckv_cache.data_ptr(), w.kpe_cache.data_ptr(),
        w.sparse_indices.data_ptr(), w.num_tokens, w.num_pages, w.sm_scale, out.data_ptr(), lse.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def _oracle(w, tokens):
    idx = w.sparse_indices[tokens]
    ckv, kpe, idx_c = compact_pool(w.ckv_cache, w.kpe_cache, idx)
    return sparse_attention_oracle(w.q_nope[tokens].cpu(), w.q_pe[tokens].cpu(), ckv.cpu(), kpe.cpu(),
                                   idx_c.cpu(), w.sm_scale)


def test_noalloc_matches_workspace_entry_point_and_oracle_on_three_calls():
    dsa = pkg()
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    W = submodule("workloads")
    # a plan where every token spans many CTAs, one where CTAs span several
    # tokens (both go through the merge of split tokens), then the first again
    small = W.make_uniform(5, 64, seed=31, device="cuda", pad=300)
    large = W.config2(device="cuda", num_tokens=200, pool_pages=4096)
    for w, tokens in ((small, list(range(5))), (large, [0, 1, 2, 57, 99, 100, 150, 199]),
                      (small, list(range(5)))):
        ref_out, ref_lse = dsa.kernel(*w.args())
        out = torch.full_like(ref_out, float("nan"))
        lse = torch.full_like(ref_lse, float("nan"))
        st = _noalloc(lib, w, out, lse)
        assert st == lib_mod.DSA_OK, lib_mod.status_string(st)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out), "output differs from the workspace entry point"
        assert torch.equal(lse, ref_lse), "lse differs from the workspace entry point"
        o_ref, l_ref = _oracle(w, tokens)
        assert_output_close(out[tokens], o_ref)
        assert_lse_close(lse[tokens], l_ref)


def test_noalloc_rejects_bad_arguments_without_device_work():
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    assert lib.dsa_sparse_attention_fwd_noalloc(None, None, None, None, None, -1, 1, 0.1, None, None, None) \
        == lib_mod.DSA_ERR_INVALID_ARGUMENT
    assert lib.dsa_sparse_attention_fwd_noalloc(None, None, None, None, None, 0, 1, 0.1, None, None, None) \
        == lib_mod.DSA_OK
    # a valid count with unusable pointers is rejected by the host checks
    assert lib.dsa_sparse_attention_fwd_noalloc(16, 16, 16, 16, 16, 4, 1, 0.1, 16, 16, None) \
        == lib_mod.DSA_ERR_INVALID_ARGUMENT


def _read(lib, lib_mod):
    import ctypes
    flags = ctypes.c_uint32(0)
    st = lib.dsa_sparse_attention_noalloc_read_errors(torch.cuda.current_stream().cuda_stream, ctypes.byref(flags))
    return st, flags.value


def test_noalloc_device_findings_are_readable():
    """A bad index, then a pipeline wait that runs out (the test hook: every
    CTA waits for a word nothing sets, under a 1 ms limit): each is reported by
    dsa_sparse_attention_noalloc_read_errors, the read clears it, and the next
    call is bitwise the workspace entry point's."""
    dsa = pkg()
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    W = submodule("workloads")
    w = W.make_uniform(4, 40, seed=41, device="cuda")
    out = torch.empty((4, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((4, 16), dtype=torch.float32, device="cuda")
    assert _noalloc(lib, w, out, lse) == lib_mod.DSA_OK
    assert _read(lib, lib_mod)[0] == lib_mod.DSA_OK
    bad = W.Workload(w.name, w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, w.sparse_indices.clone(), w.sm_scale)
    bad.sparse_indices[1, 7] = 40 * 64   # one past the pool
    assert _noalloc(lib, bad, out, lse) == lib_mod.DSA_OK
    st, flags = _read(lib, lib_mod)
    assert st == lib_mod.DSA_ERR_BAD_INDEX and flags != 0
    assert _read(lib, lib_mod)[0] == lib_mod.DSA_OK   # the read cleared it
    try:
        assert lib.dsa_sparse_attention_set_wait_timeout_ns(1_000_000) == lib_mod.DSA_OK
        assert lib.dsa_sparse_attention_test_hold(1) == lib_mod.DSA_OK
        assert _noalloc(lib, w, out, lse) == lib_mod.DSA_OK
        torch.cuda.synchronize()
    finally:
        assert lib.dsa_sparse_attention_test_hold(0) == lib_mod.DSA_OK
        assert lib.dsa_sparse_attention_set_wait_timeout_ns(0) == lib_mod.DSA_OK
    assert _read(lib, lib_mod)[0] == lib_mod.DSA_ERR_DEVICE_TIMEOUT
    ref_out, ref_lse = dsa.kernel(*w.args())
    assert _noalloc(lib, w, out, lse) == lib_mod.DSA_OK
    assert _read(lib, lib_mod)[0] == lib_mod.DSA_OK
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
