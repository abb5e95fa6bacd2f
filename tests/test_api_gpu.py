"""The Python entry points mirror the reference's interface and error
behaviour (solution/cuda/kernel.cu:673-729): DPS writes in place, the
value-returning form allocates, bad arguments raise, N=0 is a no-op."""
import pytest
import torch

from tests.conftest import submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")


def test_dps_writes_in_place(dsa):
    w = W.make_uniform(3, 40, seed=2, device="cuda")
    out = torch.full((3, 16, 512), 7.0, dtype=torch.bfloat16, device="cuda")
    lse = torch.full((3, 16), 7.0, dtype=torch.float32, device="cuda")
    ptr_o, ptr_l = out.data_ptr(), lse.data_ptr()
    dsa.launch_sparse_attention_c(*w.args(), out, lse)
    o2, l2 = dsa.kernel(*w.args())
    torch.cuda.synchronize()
    assert out.data_ptr() == ptr_o and lse.data_ptr() == ptr_l
    assert torch.equal(out, o2) and torch.equal(lse, l2)


def test_zero_tokens_is_noop(dsa):
    w = W.make_uniform(0, 4, seed=1, device="cuda")
    out, lse = dsa.kernel(*w.args())
    assert out.shape == (0, 16, 512) and lse.shape == (0, 16)


def test_sm_scale_as_tensor_or_float(dsa):
    w = W.make_uniform(2, 40, seed=4, device="cuda")
    a = dsa.kernel(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, w.sparse_indices, w.sm_scale)
    b = dsa.kernel(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, w.sparse_indices,
                   torch.tensor(w.sm_scale, dtype=torch.float32))
    torch.cuda.synchronize()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("mutate", ["dtype", "shape", "noncontig", "cpu", "idx_dtype", "out_shape"])
def test_bad_arguments_raise(dsa, mutate):
    w = W.make_uniform(2, 40, seed=4, device="cuda")
    args = list(w.args())
    out = torch.empty((2, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((2, 16), dtype=torch.float32, device="cuda")
    if mutate == "dtype":
        args[0] = args[0].float()
    elif mutate == "shape":
        args[1] = args[1][:, :8]
    elif mutate == "noncontig":
        args[2] = args[2].transpose(1, 2)
    elif mutate == "cpu":
        args[3] = args[3].cpu()
    elif mutate == "idx_dtype":
        args[4] = args[4].long()
    elif mutate == "out_shape":
        out = out[:1]
    with pytest.raises(dsa.DsaError):
        dsa.launch_sparse_attention_c(*args, out, lse)


def test_capi_rejects_host_pointers(dsa):
    """The C ABI itself refuses memory that is not on the current device."""
    lib_mod = submodule("_lib")
    lib = lib_mod.load()
    w = W.make_uniform(2, 40, seed=4, device="cuda")
    host_q = w.q_nope.cpu().pin_memory()
    out = torch.empty((2, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((2, 16), dtype=torch.float32, device="cuda")
    ws = dsa.workspace_for(torch.device("cuda", 0), 2)
    st = lib.dsa_sparse_attention_fwd(host_q.data_ptr(), w.q_pe.data_ptr(), w.ckv_cache.data_ptr(),
                                      w.kpe_cache.data_ptr(), w.sparse_indices.data_ptr(), 2, 40, 0.1,
                                      out.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), None)
    assert st == lib_mod.DSA_ERR_INVALID_ARGUMENT
    st = lib.dsa_sparse_attention_fwd(w.q_nope.data_ptr(), w.q_pe.data_ptr(), w.ckv_cache.data_ptr(),
                                      w.kpe_cache.data_ptr(), w.sparse_indices.data_ptr(), 2, 40, 0.1,
                                      out.data_ptr(), lse.data_ptr(), ws.data_ptr(), 1024, None)
    assert st == lib_mod.DSA_ERR_WORKSPACE_TOO_SMALL


def test_runs_on_side_stream(dsa):
    w = W.make_uniform(5, 40, seed=9, device="cuda")
    ref = dsa.kernel(*w.args())
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        got = dsa.kernel(*w.args())
    s.synchronize()
    assert torch.equal(ref[0], got[0]) and torch.equal(ref[1], got[1])


def test_calls_take_the_cpp_fast_path(dsa, monkeypatch):
    """Calls on the current stream go through the C++ fast path (its checks,
    then the C ABI), with bitwise the results of the Python-checked path."""
    att = submodule("attention")
    host = att._load_host()
    assert host, "the C++ fast path is not built"
    w = W.make_uniform(3, 40, seed=11, device="cuda")
    calls = []
    real = host.fwd
    monkeypatch.setattr(host, "fwd", lambda *a: calls.append(1) or real(*a))
    fast = dsa.kernel(*w.args())
    assert calls, "the call did not take the C++ fast path"
    monkeypatch.setattr(att, "_host", False)   # the Python-checked path
    checked = dsa.kernel(*w.args())
    torch.cuda.synchronize()
    assert torch.equal(fast[0], checked[0]) and torch.equal(fast[1], checked[1])
