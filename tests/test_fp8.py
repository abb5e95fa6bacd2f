"""FP8 KV cache format (CPU): the quantiser's layout and accuracy, and the
library's dequantiser against the oracle's restatement of the format."""
import torch

from oracle.dsa_oracle import dequantize_kv_fp8 as oracle_dequant
from tests.conftest import submodule

fp8 = submodule("fp8")
W = submodule("workloads")


def test_layout_and_scales():
    w = W.make_uniform(2, 6, seed=21)
    ckv, kpe = w.ckv_cache, w.kpe_cache
    ckv[1, 3, 128:256] = 0          # a zero group: scale 1, values 0
    kv = fp8.quantize_kv_fp8(ckv, kpe)
    assert kv.dtype == torch.uint8 and tuple(kv.shape) == (6, 64, 656)
    scales = kv[..., 512:528].contiguous().view(torch.float32)
    amax = ckv.float().reshape(6, 64, 4, 128).abs().amax(-1)
    expect = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    assert torch.equal(scales, expect)
    assert torch.equal(kv[..., 528:], kpe.contiguous().view(torch.uint8).reshape(6, 64, 128))
    d_ckv, d_kpe = fp8.dequantize_kv_fp8(kv)
    assert torch.all(d_ckv[1, 3, 128:256] == 0)
    assert torch.equal(d_kpe, kpe)


def test_dequantiser_matches_oracle_and_error_is_bounded():
    w = W.make_uniform(2, 16, seed=22)
    kv = fp8.quantize_kv_fp8(w.ckv_cache, w.kpe_cache)
    ckv_l, kpe_l = fp8.dequantize_kv_fp8(kv)
    ckv_o, kpe_o = oracle_dequant(kv)
    assert torch.equal(ckv_l, ckv_o) and torch.equal(kpe_l, kpe_o)
    # e4m3 keeps 3 mantissa bits: |error| <= 2^-4 |x| for normal values, and
    # at most half the smallest subnormal step (2^-10 * scale) below them
    x = w.ckv_cache.float().reshape(16, 64, 4, 128)
    scale = kv[..., 512:528].contiguous().view(torch.float32)[..., None]
    err = (ckv_o.float().reshape(16, 64, 4, 128) - x).abs()
    bound = torch.maximum(x.abs() * 2.0 ** -4, scale * 2.0 ** -10) * 1.02 + x.abs() * 2.0 ** -8
    assert torch.all(err <= bound)
    # the largest value of each group is represented exactly (448 * scale)
    assert torch.allclose(ckv_o.float().reshape(16, 64, 4, 128).abs().amax(-1), x.abs().amax(-1), rtol=2 ** -8)
