import importlib
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

PKG_NAME = "karnbirkhera-mlsys2026-dsa_sparse_attention_b200"

# Contest tolerance (FAQ.md:104-110): an output element fails only if BOTH its
# absolute and its relative error exceed 1e-2; the lse must match to 1e-3.
OUT_ATOL = 1e-2
OUT_RTOL = 1e-2
LSE_ATOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pkg():
    return importlib.import_module(PKG_NAME)


def submodule(name):
    return importlib.import_module(f"{PKG_NAME}.{name}")


def assert_output_close(out, ref, atol=OUT_ATOL, rtol=OUT_RTOL):
    """Contest rule: element fails iff |d| > atol and |d| > rtol*|ref|."""
    import torch
    out = out.float().cpu()
    ref = ref.float().cpu()
    d = (out - ref).abs()
    bad = (d > atol) & (d > rtol * ref.abs())
    nbad = int(bad.sum().item())
    assert nbad == 0, f"{nbad} of {bad.numel()} output elements out of tolerance; max abs err {d.max().item():.3e}"


def assert_lse_close(lse, ref, atol=LSE_ATOL):
    import torch
    lse = lse.float().cpu()
    ref = ref.float().cpu()
    inf_ref = torch.isinf(ref)
    assert torch.equal(torch.isinf(lse), inf_ref), "lse -inf pattern differs"
    if (~inf_ref).any():
        d = (lse[~inf_ref] - ref[~inf_ref]).abs().max().item()
        assert d <= atol, f"lse max abs err {d:.3e} > {atol}"


@pytest.fixture(scope="session")
def dsa():
    return pkg()
