"""flashinfer-bench packaging on the GPU: the unpacked solutions' kernel.py,
compiled from the packed sources, gives bitwise the library's results."""
import importlib.util

import pytest
import torch

from tests.conftest import submodule

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


def test_packed_indexer_matches_library(dsa, tmp_path, monkeypatch):
    mod = load_packed("indexer", tmp_path, monkeypatch)
    w = W.indexer_small(device="cuda")
    out = torch.empty((w.batch, 2048), dtype=torch.int32, device="cuda")
    mod.launch_topk_c(w.q_index_fp8.view(torch.float8_e4m3fn), *w.args()[1:], out)
    ref = dsa.topk_indexer(*w.args())
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
