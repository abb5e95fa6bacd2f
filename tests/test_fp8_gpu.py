"""GPU parity of the FP8 KV cache variant (dsa_sparse_attention_fwd_fp8).

The FP8 path dequantises each gathered row in shared memory to exactly the
bf16 values dequantize_kv_fp8 gives, then runs the bf16 pipeline unchanged, so
its results must be BITWISE equal to the bf16 operator on the dequantised
cache; against the oracle they are held to the contest tolerance (output fails
iff |err| > 1e-2 and |err| > 1e-2 |ref|; lse within 1e-3).
"""
import ctypes

import pytest
import torch

from oracle.dsa_oracle import compact_pool, sparse_attention_fp8_oracle
from tests.conftest import assert_lse_close, assert_output_close, submodule

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

W = submodule("workloads")
fp8 = submodule("fp8")


def both(dsa, w, idx=None):
    """(fp8 result, bf16 result on the dequantised cache) on the same indices."""
    idx = w.sparse_indices if idx is None else idx
    kv = fp8.quantize_kv_fp8(w.ckv_cache, w.kpe_cache)
    out8, lse8 = dsa.kernel_fp8(w.q_nope, w.q_pe, kv, idx, w.sm_scale)
    ckv_d, kpe_d = fp8.dequantize_kv_fp8(kv)
    out, lse = dsa.kernel(w.q_nope, w.q_pe, ckv_d, kpe_d, idx, w.sm_scale)
    torch.cuda.synchronize()
    assert dsa.check_device_errors() == 0
    return (out8, lse8), (out, lse), kv


def oracle_on(w, kv, tokens=None):
    sel = slice(None) if tokens is None else tokens
    idx = w.sparse_indices[sel]
    used = torch.unique(idx[idx >= 0] // 64)
    remap = torch.full((kv.shape[0],), -1, dtype=torch.int64, device=idx.device)
    remap[used] = torch.arange(used.numel(), device=idx.device)
    idx_c = torch.where(idx >= 0, remap[(idx.clamp(min=0) // 64)] * 64 + idx % 64, idx).to(torch.int32)
    return sparse_attention_fp8_oracle(w.q_nope[sel].cpu(), w.q_pe[sel].cpu(), kv[used].cpu(), idx_c.cpu(),
                                       w.sm_scale)


@pytest.mark.parametrize("n", [1, 4, 9, 17, 64, 149])
def test_fp8_equals_bf16_on_dequantised_cache(dsa, n):
    w = W.make_uniform(n, 40, seed=3000 + n, device="cuda", pad=(n * 41) % 300)
    (o8, l8), (o, l), kv = both(dsa, w)
    assert torch.equal(o8, o) and torch.equal(l8, l)
    ro, rl = oracle_on(w, kv)
    assert_output_close(o8, ro)
    assert_lse_close(l8, rl)


def test_fp8_masking_and_duplicates(dsa):
    n = 24
    w = W.make_uniform(n, 64, seed=78, device="cuda")
    idx = w.sparse_indices
    idx[0] = -1
    idx[1, 1:] = -1
    idx[2, :-1] = -1
    idx[3, ::2] = -1
    idx[4, 128:1920] = -1
    idx[6:12] = -1
    idx[13, 512:1024] = idx[13, :512]
    (o8, l8), (o, l), kv = both(dsa, w)
    assert torch.equal(o8, o) and torch.equal(l8, l)
    ro, rl = oracle_on(w, kv)
    assert_output_close(o8, ro)
    assert_lse_close(l8, rl)
    assert torch.all(o8[0] == 0) and torch.all(torch.isneginf(l8[0]))


def test_fp8_config2_full_size(dsa):
    """Benchmark config 2 with its pool quantised (1.38 GB of 656-byte rows)."""
    w = W.config2(device="cuda")
    (o8, l8), (o, l), kv = both(dsa, w)
    assert torch.equal(o8, o) and torch.equal(l8, l)
    sel = torch.arange(0, 64, 7)
    ro, rl = oracle_on(w, kv, sel)
    assert_output_close(o8[sel], ro)
    assert_lse_close(l8[sel], rl)


def test_fp8_paged_equals_slot_ids(dsa):
    w = W.config2(device="cuda")
    kv = fp8.quantize_kv_fp8(w.ckv_cache, w.kpe_cache)
    out_p, lse_p = dsa.kernel_fp8_paged(w.q_nope, w.q_pe, kv, w.meta["block_table"], w.meta["positions"],
                                        w.sm_scale)
    out_s, lse_s = dsa.kernel_fp8(w.q_nope, w.q_pe, kv, w.sparse_indices, w.sm_scale)
    torch.cuda.synchronize()
    assert dsa.check_device_errors() == 0
    assert torch.equal(out_p, out_s) and torch.equal(lse_p, lse_s)


def test_fp8_bad_indices_reported_and_masked(dsa):
    w = W.make_uniform(4, 40, seed=31, device="cuda")
    kv = fp8.quantize_kv_fp8(w.ckv_cache, w.kpe_cache)
    idx = w.sparse_indices.clone()
    idx[1, 5] = 40 * 64            # one past the pool
    idx[2, 7] = -3
    out, lse = dsa.kernel_fp8(w.q_nope, w.q_pe, kv, idx, w.sm_scale)
    torch.cuda.synchronize()
    with pytest.raises(dsa.DsaError) as ei:
        dsa.check_device_errors()
    assert "BAD_INDEX" in str(ei.value)
    masked = idx.clone()
    masked[1, 5] = -1
    masked[2, 7] = -1
    ref_out, ref_lse = dsa.kernel_fp8(w.q_nope, w.q_pe, kv, masked, w.sm_scale)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)


def test_fp8_capi_rejects_bad_arguments(dsa):
    lib = submodule("_lib").load()
    w = W.make_uniform(2, 8, seed=32, device="cuda")
    kv = fp8.quantize_kv_fp8(w.ckv_cache, w.kpe_cache)
    out = torch.empty((2, 16, 512), dtype=torch.bfloat16, device="cuda")
    lse = torch.empty((2, 16), dtype=torch.float32, device="cuda")
    ws = dsa.workspace_for(torch.device("cuda"), 2)
    base = [w.q_nope.data_ptr(), w.q_pe.data_ptr(), kv.data_ptr(), w.sparse_indices.data_ptr(), 2, 8,
            w.sm_scale, out.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), None]
    assert lib.dsa_sparse_attention_fwd_fp8(*base) == 0
    bad = list(base)
    bad[2] = None
    assert lib.dsa_sparse_attention_fwd_fp8(*bad) == 1
    bad = list(base)
    bad[2] = kv.data_ptr() + 8
    assert lib.dsa_sparse_attention_fwd_fp8(*bad) == 1
    torch.cuda.synchronize()
