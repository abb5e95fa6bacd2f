"""Same-box comparison with the reference's own optimised CUDA kernel.

oracle/build_ref_cuda.py compiles the reference's shipped solution
(solution/cuda/kernel.cu) unchanged for sm_100a into oracle/_ref/.  On the GPU
this file checks, on config 1 and on uniform shapes with num_tokens = 1, 2, 4,
6, 8 (the reference kernel rejects num_tokens >= 9, kernel.cu:688-691), with
and without -1 padding:

  * that kernel against oracle/dsa_oracle.py:reference_cuda_oracle, a CPU
    restatement of ITS algorithm (splits, per-split online softmax, fused
    reduce) — this pins the restatement on the reference's GPU output;
  * where the kernel has at most 32 splits per token (num_tokens >= 5), that
    kernel against the operator's oracle (the naive kernel's semantics), and
    the library against that kernel;
  * for every shape, the library against the operator's oracle.

The reference kernel does not compute the operator when it uses more than 32
splits per token (num_tokens <= 4: S = 33 or 64): its reduce reads the
per-split statistics with one lane per split over 32 lanes, so splits 32..
are left out of l and lse and mis-weighted in the output (kernel.cu:439-475).
Only valid inputs are given to the reference kernel: its barrier waits spin
without a bound (kernel.cu:105-116) and its copies read any index >= 0
unchecked.
"""
import pytest
import torch

from oracle.build_ref_cuda import MAX_TOKENS, load_ref_cuda
from oracle.dsa_oracle import reference_cuda_oracle, reference_cuda_splits, sparse_attention_oracle
from tests.conftest import assert_lse_close, assert_output_close, submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")


@pytest.fixture(scope="module")
def ref():
    mod = load_ref_cuda()
    if mod is None:
        pytest.skip("oracle/_ref/dsa_ref_cuda.so not built (needs the reference tree at build time)")
    return mod


def run_ref(ref, w):
    n = w.num_tokens
    out = torch.empty((n, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((n, 16), dtype=torch.float32, device="cuda")
    ref.launch_sparse_attention_c(*w.args()[:5], float(w.sm_scale), out, lse)
    torch.cuda.synchronize()
    return out, lse


CASES = [("config1", lambda: W.config1(device="cuda"))] + [
    (f"uniform_n{n}_pad{pad}", (lambda n=n, pad=pad: W.make_uniform(n, 64, seed=700 + n + pad, device="cuda",
                                                                     pad=pad)))
    for n in (1, 2, 4, 6, 8) for pad in (0, 517)]


@pytest.mark.parametrize("name,make", CASES, ids=[c[0] for c in CASES])
def test_reference_cuda_kernel_and_library(dsa, ref, name, make):
    w = make()
    assert w.num_tokens <= MAX_TOKENS
    assert int(w.sparse_indices.max()) < w.num_pages * 64 and int(w.sparse_indices.min()) >= -1
    cpu = [t.cpu() for t in w.args()[:5]]
    r_out, r_lse = run_ref(ref, w)
    # the reference kernel computes its own algorithm (restated on CPU)
    a_out, a_lse = reference_cuda_oracle(*cpu, w.sm_scale)
    assert_output_close(r_out, a_out)
    assert_lse_close(r_lse, a_lse)
    o_out, o_lse = sparse_attention_oracle(*cpu, w.sm_scale)
    out, lse = dsa.kernel(*w.args())
    torch.cuda.synchronize()
    assert dsa.check_device_errors() == 0
    assert_output_close(out, o_out)
    assert_lse_close(lse, o_lse)
    if reference_cuda_splits(w.num_tokens) <= 32:
        # where its reduce is the exact split-KV combine, it computes the operator
        assert_output_close(r_out, o_out)
        assert_lse_close(r_lse, o_lse)
        assert_output_close(out, r_out)
        assert_lse_close(lse, r_lse)
