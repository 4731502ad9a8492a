"""GPU parity of the union launch of the pair family: blocks of 128 / H
queries (H = 16, 32, 64) run as 128-row items over the union of their
selected keys, one membership mask per query and tile (duplicate slots as
repeated entries).

Selected explicitly with ``Tuning(bm=16, bn=32, split=1, pv_cols=128)`` and
checked against the CPU oracle with the benchmark gates on the reference's
index families, ragged TOPK, key ranges spanning several build passes, many
blocks per cluster, blocks without a valid index, and sampled rows of
prefill_tp8.
"""
import pytest
import torch

import bench
import dsa_b200
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu

UNION = dsa_b200.Tuning(16, 32, 1, pv_cols=128)


def _run(data):
    out = dsa_b200.forward(*[t.cuda() for t in data], config=UNION)
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0, "a bounded device-side wait timed out"
    return out


def _check(got, ref):
    metrics = oracle.accuracy([t.float().cpu() for t in got], ref)
    assert oracle.passes(metrics), metrics
    return metrics


@pytest.mark.parametrize("heads,queries", [(16, 16), (32, 8), (64, 4)])
@pytest.mark.parametrize("family", oracle.FAMILIES)
def test_union_families(cuda_lib, heads, queries, family):
    shape = (2, queries, heads, 1024, 256)
    data = oracle.make_inputs(shape, 20261103, family)
    _check(_run(data), oracle.reference_forward(*data))


@pytest.mark.parametrize("length,topk", [(3000, 1), (3000, 33), (3000, 100), (9000, 2048), (40000, 512)])
def test_union_tails_and_passes(cuda_lib, length, topk):
    shape = (1, 16, 16, length, topk)
    data = oracle.make_inputs(shape, 5, "normal")
    _check(_run(data), oracle.reference_forward(*data))


def test_union_many_blocks(cuda_lib):
    """More blocks than resident clusters: every cluster loops over items."""
    shape = (1, 1024, 16, 2048, 512)
    data = oracle.make_inputs(shape, 11, "uniform")
    _check(_run(data), oracle.reference_forward(*data))


def test_union_block_without_valid_index(cuda_lib):
    shape = (1, 16, 16, 1024, 64)
    q, kv, qr, kr, ids = oracle.make_inputs(shape, 7, "normal")
    ids[0, :8] = -1  # the whole first block of 8 queries
    ids[0, 9] = 5000  # one more query with only invalid indices
    out, mx, sm = _run((q, kv, qr, kr, ids))
    ref = oracle.reference_forward(q, kv, qr, kr, ids, defined_invalid=True)
    empty = torch.zeros((1, 16), dtype=torch.bool)
    empty[0, :8] = True
    empty[0, 9] = True
    out, mx, sm = out.float().cpu(), mx.cpu(), sm.cpu()
    assert torch.equal(out[empty], torch.zeros_like(out[empty]))
    assert bool(torch.isneginf(mx[:, 0][empty]).all()) and torch.equal(sm[:, 0][empty], torch.zeros_like(sm[:, 0][empty]))
    keep = ~empty
    got = (out[keep].unsqueeze(1), mx[:, 0][keep].unsqueeze(1).unsqueeze(1), sm[:, 0][keep].unsqueeze(1).unsqueeze(1))
    want = (ref[0][keep].unsqueeze(1), ref[1][:, 0][keep].unsqueeze(1).unsqueeze(1),
            ref[2][:, 0][keep].unsqueeze(1).unsqueeze(1))
    _check(got, want)


def test_union_matches_stream_family(cuda_lib):
    shape = (1, 256, 16, 8192, 2048)
    data = [t.cuda() for t in oracle.make_inputs(shape, 3, "normal")]
    a = dsa_b200.forward(*data, config=dsa_b200.Tuning(16, 32, 1))
    b = dsa_b200.forward(*data, config=UNION)
    torch.cuda.synchronize()
    m = oracle.accuracy([t.float().cpu() for t in b], [t.float().cpu() for t in a])
    # both outputs are BF16-rounded results, each within 5e-3 of the FP32
    # oracle (small values at 16 heads: one BF16 ulp is ~0.7 % of the max),
    # so they agree within twice that; the maxima are FP32 (accumulation
    # order only)
    assert m["output"]["max_normalized"] < 1e-2 and m["maximum"]["max_normalized"] < 1e-5, m


def test_union_prefill_tp8(cuda_lib):
    shape = bench.CONFIGS["prefill_tp8"]
    data = bench.make_device_inputs(shape, bench.SEED, "uniform", "cuda")
    out, mx, sm = dsa_b200.forward(*data, config=UNION)
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    b, s, h, _, _ = shape
    assert bool(torch.isfinite(out.float()).all()) and bool((sm >= 1.0 - 1e-6).all())
    rows = list(range(0, b * s, 37)) + [b * s - 1]
    ref = oracle.reference_forward(*bench.compact_for_oracle(data, rows))
    rows_t = torch.as_tensor(rows, device="cuda")
    got = (out.reshape(b * s, h, 512)[rows_t].unsqueeze(1),
           mx.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h),
           sm.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h))
    _check(got, ref)


@pytest.mark.parametrize("name", ["prefill_b4_h64", "prefill_b4_h32"])
def test_default_union_launch_for_32_and_64_heads(cuda_lib, name):
    """The shape heuristic runs dense 32- and 64-head prefill (B=4,
    SQ=8192, L=8192, TOPK=2048) on the union launch; sampled rows against
    the oracle."""
    shape = dsa_b200.CASE_SHAPES[name]
    data = bench.make_device_inputs(shape, bench.SEED, "uniform", "cuda")
    (out, mx, sm), kernels = dsa_b200.forward(*data, return_kernels=True)
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    assert [k.name for k in kernels] == ["dsa_union_build", "dsa_fwd_pair_union"], kernels
    b, s, h, _, _ = shape
    rows = list(range(0, b * s, 331)) + [b * s - 1]
    ref = oracle.reference_forward(*bench.compact_for_oracle(data, rows))
    rows_t = torch.as_tensor(rows, device="cuda")
    got = (out.reshape(b * s, h, 512)[rows_t].unsqueeze(1),
           mx.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h),
           sm.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h))
    _check(got, ref)
