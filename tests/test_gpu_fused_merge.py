"""Split merges inside the main kernel (one launch per call).

Split-V family, split S in 2..16: the S CTAs of one (token, value half) run
as one thread-block cluster and merge their FP32 partials themselves (the
merge of dsa/merge.py:13-91: m = max m_s, w_s = exp(m_s - m),
l = sum w_s l_s, O = sum w_s O_s / l): partials through the L2, row
statistics through distributed shared memory when S divides 128 (else the
L2), one cluster barrier. Stream family, split 2..8: the split CTAs of one
(token, 16-head group) form the cluster and merge the same way after one
cluster barrier. No separate merge kernel runs. Checked against the CPU
oracle with the parity gates, including splits whose keys are all masked and
rows without a valid index.
"""
import pytest
import torch

import bench
import dsa_b200
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu


def _split_v(split):
    return dsa_b200.Tuning(128, 32, split, pv_cols=256)


def _run(data, split):
    (out, mx, sm), kernels = dsa_b200.forward(*[t.cuda() for t in data], config=_split_v(split),
                                              return_kernels=True)
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    return (out, mx, sm), kernels


def _check(got, ref):
    metrics = oracle.accuracy([t.float().cpu() for t in got], ref)
    assert oracle.passes(metrics), metrics


@pytest.mark.parametrize("split", [2, 3, 4, 5, 7, 8, 12, 16])
def test_fused_merge_matches_oracle(cuda_lib, split):
    shape = (2, 2, 128, 8192, 2048)
    data = oracle.make_inputs(shape, 20261103, "normal")
    out, kernels = _run(data, split)
    assert [k.name for k in kernels] == ["dsa_fwd_umma"], kernels
    _check(out, oracle.reference_forward(*data))


@pytest.mark.parametrize("split", [4, 16])
def test_fused_merge_all_masked_splits(cuda_lib, split):
    """The second half of every query's indices is -1 (the reference's
    "invalid" family): splits there hold no valid key and merge with weight 0."""
    shape = (1, 3, 128, 4096, 1024)
    data = oracle.make_inputs(shape, 20261102, "invalid")
    out, _ = _run(data, split)
    _check(out, oracle.reference_forward(*data))


@pytest.mark.parametrize("split", [2, 8])
def test_fused_merge_row_without_valid_index(cuda_lib, split):
    shape = (1, 3, 128, 1024, 512)
    q, kv, qr, kr, ids = oracle.make_inputs(shape, 11, "duplicates")
    ids[0, 1] = -1
    data = (q, kv, qr, kr, ids)
    (out, mx, sm), _ = _run(data, split)
    ref = oracle.reference_forward(*data, defined_invalid=True)
    out, mx, sm = out.float().cpu(), mx.cpu(), sm.cpu()
    assert torch.equal(out[0, 1], torch.zeros_like(out[0, 1]))
    assert bool(torch.isneginf(mx[0, 0, 1]).all()) and torch.equal(sm[0, 0, 1], torch.zeros_like(sm[0, 0, 1]))
    keep = [0, 2]
    _check((out[:, keep], mx[:, :, keep], sm[:, :, keep]), (ref[0][:, keep], ref[1][:, :, keep], ref[2][:, :, keep]))


@pytest.mark.parametrize("name,split", [("decode_b1", 16), ("decode_b8", 4), ("decode_b8", 16)])
def test_fused_merge_benchmark_configs(cuda_lib, name, split):
    """decode_b8 with split 16 launches 512 CTAs in clusters of 16: more
    clusters than fit at once, so they run in several waves."""
    shape = bench.CONFIGS[name]
    data = bench.make_device_inputs(shape, bench.SEED, "uniform", "cuda")
    (out, mx, sm), kernels = dsa_b200.forward(*data, config=_split_v(split), return_kernels=True)
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0 and len(kernels) == 1
    b, s, h, _, _ = shape
    rows = list(range(b * s))
    ref = oracle.reference_forward(*bench.compact_for_oracle(data, rows))
    got = (out.reshape(b * s, 1, h, 512), mx.reshape(b * s, 1, 1, h), sm.reshape(b * s, 1, 1, h))
    _check(got, ref)


def test_default_decode_launch_is_one_kernel(cuda_lib):
    """The shape-keyed default for few-query H = 128 shapes picks a split the
    cluster merge takes: one kernel per call."""
    for name in ("decode_b1", "decode_b8"):
        shape = bench.CONFIGS[name]
        data = bench.make_device_inputs(shape, bench.SEED, "uniform", "cuda")
        _, kernels = dsa_b200.forward(*data, return_kernels=True)
        torch.cuda.synchronize()
        assert [k.name for k in kernels] == ["dsa_fwd_umma"], (name, kernels)


@pytest.mark.parametrize("split", [2, 3, 4, 8])
def test_stream_cluster_merge(cuda_lib, split):
    """The stream family (16-head groups) with splits 2..8: one kernel, the
    reference's "invalid" family (splits without a valid key) and a query
    without any valid index (output 0, max -inf, sum 0)."""
    shape = (2, 2, 32, 4096, 1024)
    q, kv, qr, kr, ids = oracle.make_inputs(shape, 20261104, "invalid")
    ids[1, 0] = -1
    data = (q, kv, qr, kr, ids)
    (out, mx, sm), kernels = dsa_b200.forward(*[t.cuda() for t in data], config=dsa_b200.Tuning(16, 32, split),
                                              return_kernels=True)
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    assert [k.name for k in kernels] == ["dsa_fwd_stream"], kernels
    ref = oracle.reference_forward(*data, defined_invalid=True)
    out, mx, sm = out.float().cpu(), mx.cpu(), sm.cpu()
    assert torch.equal(out[1, 0], torch.zeros_like(out[1, 0]))
    assert bool(torch.isneginf(mx[1, 0, 0]).all()) and torch.equal(sm[1, 0, 0], torch.zeros_like(sm[1, 0, 0]))
    for b, t in ((0, 0), (0, 1), (1, 1)):
        _check((out[b:b + 1, t:t + 1], mx[b:b + 1, :, t:t + 1], sm[b:b + 1, :, t:t + 1]),
               (ref[0][b:b + 1, t:t + 1], ref[1][b:b + 1, :, t:t + 1], ref[2][b:b + 1, :, t:t + 1]))
