"""flashinfer-bench packaging on the GPU: the unpacked solutions' kernel.py,
compiled from the packed sources, gives bitwise the library's results and
matches the CPU oracles (contest tolerance for the attention; the indexer's
selections up to near-ties at the boundary); its argument checks reject a
wrong dtype, shape or alignment before any device work."""
import importlib.util

import pytest
import torch

from oracle.dsa_indexer_oracle import topk_indexer_oracle
from oracle.dsa_oracle import sparse_attention_oracle
from tests.conftest import assert_lse_close, assert_output_close, submodule
from tests.test_indexer_gpu import check_rows

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

pack = submodule("fib.pack")
W = submodule("workloads")


def load_packed(which, tmp_path, monkeypatch):
    sol_dir = tmp_path / which
    pack.unpack(pack.solution(which), str(sol_dir))
    monkeypatch.setenv("DSA_FIB_CACHE", str(tmp_path / "cache"))
    spec = importlib.util.spec_from_file_location(f"dsa_fib_kernel_{which}", str(sol_dir / "kernel.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_packed_attention_matches_library(dsa, tmp_path, monkeypatch):
    mod = load_packed("attention", tmp_path, monkeypatch)
    w = W.config1(device="cuda")
    out = torch.empty((w.num_tokens, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((w.num_tokens, 16), dtype=torch.float32, device="cuda")
    mod.launch_sparse_attention_c(*w.args(), out, lse)
    ref_out, ref_lse = dsa.kernel(*w.args())
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
    o_ref, l_ref = sparse_attention_oracle(*(t.cpu() for t in w.args()[:5]), w.sm_scale)
    assert_output_close(out, o_ref)
    assert_lse_close(lse, l_ref)


def test_packed_attention_rejects_bad_arguments(tmp_path, monkeypatch):
    mod = load_packed("attention", tmp_path, monkeypatch)
    w = W.config1(device="cuda")
    n = w.num_tokens
    out = torch.empty((n, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((n, 16), dtype=torch.float32, device="cuda")
    qn, qp, ckv, kpe, idx, scale = w.args()
    with pytest.raises(ValueError, match="sparse_indices must be torch.int32"):
        mod.launch_sparse_attention_c(qn, qp, ckv, kpe, idx.long(), scale, out, lse)
    with pytest.raises(ValueError, match="q_pe must have shape"):
        mod.launch_sparse_attention_c(qn, qp[:, :8].contiguous(), ckv, kpe, idx, scale, out, lse)
    with pytest.raises(ValueError, match="lse must be torch.float32"):
        mod.launch_sparse_attention_c(qn, qp, ckv, kpe, idx, scale, out, lse.half())
    raw = torch.empty(out.numel() * 2 + 8, dtype=torch.uint8, device="cuda")
    skewed = raw[8:8 + out.numel() * 2].view(torch.bfloat16).view(out.shape)   # 8-byte aligned only
    with pytest.raises(ValueError, match="output must be 16-byte aligned"):
        mod.launch_sparse_attention_c(qn, qp, ckv, kpe, idx, scale, skewed, lse)
    with pytest.raises(ValueError, match="CUDA tensor"):
        mod.launch_sparse_attention_c(qn.cpu(), qp, ckv, kpe, idx, scale, out, lse)


def test_packed_indexer_matches_library(dsa, tmp_path, monkeypatch):
    mod = load_packed("indexer", tmp_path, monkeypatch)
    w = W.indexer_small(device="cuda")
    out = torch.empty((w.batch, 2048), dtype=torch.int32, device="cuda")
    mod.launch_topk_c(w.q_index_fp8.view(torch.float8_e4m3fn), *w.args()[1:], out)
    ref = dsa.topk_indexer(*w.args())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    ref_idx, finals = topk_indexer_oracle(*(t.cpu() for t in w.args()))
    check_rows(out, ref_idx, finals, w)   # same selections up to swaps at the boundary, descending order
