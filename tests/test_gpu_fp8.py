"""GPU parity of the FP8 KV cache forward: the kernels' dequantised rows
feed the BF16 forward; the oracle reads the same cache independently
(oracle.dequantize_kv_fp8) and runs its FP32 attention."""
import pytest
import torch

import dsa_b200
from dsa_b200 import api
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu


def _case(shape, seed, family="normal"):
    q, kv, qr, kr, ids = oracle.make_inputs(shape, seed, family)
    return q, dsa_b200.quantize_kv_fp8(kv, kr), qr, ids


def _check(got, ref):
    metrics = oracle.accuracy([t.float().cpu() for t in got], ref)
    assert oracle.passes(metrics), metrics


@pytest.mark.parametrize("heads", [16, 64, 128])
@pytest.mark.parametrize("family", ["normal", "duplicates", "invalid"])
def test_fp8_matches_oracle(cuda_lib, heads, family):
    q, cache, qr, ids = _case((2, 3, heads, 4096, 512), 20261103, family)
    out = dsa_b200.forward_fp8(*[t.cuda() for t in (q, cache, qr, ids)])
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    kv, kr = oracle.dequantize_kv_fp8(cache)
    _check(out, oracle.reference_forward(q, kv, qr, kr, ids))


def test_fp8_in_pieces(cuda_lib, monkeypatch):
    """A workspace budget of a few queries splits the call into pieces."""
    monkeypatch.setattr(api, "FP8_WORKSPACE_BUDGET", 3 * 256 * 1156)
    q, cache, qr, ids = _case((2, 7, 32, 2048, 256), 5, "peaked")
    out = dsa_b200.forward_fp8(*[t.cuda() for t in (q, cache, qr, ids)])
    torch.cuda.synchronize()
    kv, kr = oracle.dequantize_kv_fp8(cache)
    _check(out, oracle.reference_forward(q, kv, qr, kr, ids))


def test_fp8_equals_bf16_forward_on_dequantised_rows(cuda_lib):
    """Same launch family, same keys in the same order: identical results."""
    q, cache, qr, ids = _case((1, 4, 128, 8192, 2048), 3)
    kv, kr = oracle.dequantize_kv_fp8(cache)
    b, s, h, _ = q.shape
    k = ids.shape[-1]
    # the BF16 forward on the compact rows the FP8 path builds
    idx = ids.reshape(b * s, k).long()
    kv_c = kv[0, idx.clamp(0, 8191)].reshape(b * s, k, 1, 512)
    kr_c = kr[0, idx.clamp(0, 8191)].reshape(b * s, k, 1, 64)
    ids_c = torch.arange(k, dtype=torch.int32).repeat(b * s, 1).reshape(b * s, 1, 1, k)
    ref = dsa_b200.forward(*[t.cuda() for t in (q.reshape(b * s, 1, h, 512), kv_c, qr.reshape(b * s, 1, h, 64), kr_c, ids_c)])
    got = dsa_b200.forward_fp8(*[t.cuda() for t in (q, cache, qr, ids)])
    torch.cuda.synchronize()
    assert torch.equal(got[0].reshape(ref[0].shape), ref[0])
    assert torch.equal(got[1].reshape(ref[1].shape), ref[1]) and torch.equal(got[2].reshape(ref[2].shape), ref[2])
