"""The reference's own naive indexer (methodology/reference/topk_kernel_naive.cu,
compiled into oracle/_ref/ by oracle/build_ref_indexer.py) run on the GPU: it
pins the CPU oracle, and the library is checked against it directly.

Only workloads whose block tables point inside the pool are given to it (the
reference reads table entries unchecked).  Selections are compared with the
same boundary tolerance as tests/test_indexer_gpu.py: summation order differs
between the three implementations, and at::topk leaves the order of equal
scores unspecified.
"""
import pytest
import torch

from oracle.build_ref_indexer import load_ref_indexer
from oracle.dsa_indexer_oracle import topk_indexer_oracle
from tests.conftest import submodule
from tests.test_indexer_gpu import check_rows, to_dev

REF = load_ref_indexer()
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
              pytest.mark.skipif(REF is None, reason="reference indexer not built (oracle/build_ref_indexer.py)")]

W = submodule("workloads")


def run_reference(wd):
    out = torch.empty((wd.batch, 2048), dtype=torch.int32, device="cuda")
    REF.launch_topk_c(wd.q_index_fp8.view(torch.float8_e4m3fn), wd.k_index_cache, wd.weights, wd.seq_lens,
                      wd.block_table, out)
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("make", ["indexer_small", "indexer_edges", "indexer_long", "indexer_ties"])
def test_oracle_and_library_match_reference(dsa, make):
    w = getattr(W, make)()
    oracle_out, finals = topk_indexer_oracle(*w.args())
    wd = to_dev(w)
    ref_out = run_reference(wd)
    ours = dsa.topk_indexer(*wd.args())
    torch.cuda.synchronize()
    assert dsa.indexer.check_errors() == 0
    # the reference against the oracle (pins the oracle), then the library against the reference
    swaps_ref = check_rows(ref_out, oracle_out, finals, w)
    swaps_ours = check_rows(ours, ref_out, finals, w)
    if make != "indexer_ties":
        assert swaps_ref <= 4 and swaps_ours <= 4
    # rows of at most 2048 positions: every position, in both
    for b in range(w.batch):
        sl = int(w.seq_lens[b])
        if 0 < sl <= 2048:
            assert set(ref_out[b, :sl].tolist()) == set(ours.cpu()[b, :sl].tolist())
