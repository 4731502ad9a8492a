"""FP8 KV cache: the cache writer against the oracle's independent reading
of the layout (CPU); GPU parity is in test_gpu_fp8.py."""
import torch

import dsa_b200
from oracle import sparse_mla as oracle


def test_quantize_layout_round_trip():
    g = torch.Generator().manual_seed(1)
    kv = (torch.randn((2, 33, 1, 512), generator=g) * 3).bfloat16()
    kr = torch.randn((2, 33, 1, 64), generator=g).bfloat16()
    kv[0, 3] = 0  # an all-zero row: scale 1, values 0
    cache = dsa_b200.quantize_kv_fp8(kv, kr)
    assert cache.shape == (2, 33, 1, 656) and cache.dtype == torch.uint8
    dkv, dkr = oracle.dequantize_kv_fp8(cache)
    assert torch.equal(dkr, kr)
    assert torch.equal(dkv[0, 3], torch.zeros_like(dkv[0, 3]))
    # e4m3 keeps 3 mantissa bits: |error| <= 2^-4 relative, plus the BF16 rounding
    err = (dkv.float() - kv.float()).abs()
    assert bool((err <= kv.float().abs() * (2 ** -4 + 2 ** -8) + 1e-3).all())
    scales = cache[..., 512:528].contiguous().view(torch.float32)
    amax = kv.float().reshape(2, 33, 1, 4, 128).abs().amax(-1)
    expect = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    assert torch.equal(scales, expect)
