"""GPU parity of the keys family (tcgen05 with the selected keys as the MMA's
M dimension, 16 heads per CTA item, 64-key tiles).

Selected explicitly with ``Tuning(bm=16, bn=64, split=S, pv_cols=128)`` and
checked against the CPU oracle with the benchmark gates, on the index
families the reference tests (uniform, peaked, duplicates, invalid), ragged
TOPK tails, KV splits (partials + FP32 merge), several 16-head groups per
token, more work items than resident CTAs, and sampled rows of the two
16-head benchmark configs.
"""
import pytest
import torch

import bench
import dsa_b200
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu


def _tuning(split):
    return dsa_b200.Tuning(16, 64, split, pv_cols=128)


def _run(data, split):
    out = dsa_b200.forward(*[t.cuda() for t in data], config=_tuning(split))
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0, "a bounded device-side wait timed out"
    return out


def _check(got, ref):
    got = [t.float().cpu() for t in got]
    metrics = oracle.accuracy(got, ref)
    assert oracle.passes(metrics), metrics
    return metrics


@pytest.mark.parametrize("heads", [16, 32, 64])
@pytest.mark.parametrize("family", oracle.FAMILIES)
def test_keys_families(cuda_lib, heads, family):
    shape = (2, 3, heads, 4096, 256)
    data = oracle.make_inputs(shape, 20261103, family)
    _check(_run(data, 1), oracle.reference_forward(*data))


@pytest.mark.parametrize("topk,split", [(1, 1), (63, 1), (64, 1), (65, 2), (100, 1), (200, 3), (2049, 5),
                                        (2048, 32)])
def test_keys_topk_tails(cuda_lib, topk, split):
    shape = (1, 2, 16, 3000, topk)
    data = oracle.make_inputs(shape, 5, "normal")
    _check(_run(data, split), oracle.reference_forward(*data))


@pytest.mark.parametrize("split", [1, 2, 4, 7])
def test_keys_splits(cuda_lib, split):
    shape = (4, 1, 16, 8192, 2048)
    data = oracle.make_inputs(shape, 20261102, "peaked")
    _check(_run(data, split), oracle.reference_forward(*data))


def test_keys_many_items_persistent(cuda_lib):
    """More work items than resident CTAs: every CTA loops over items."""
    shape = (1, 400, 16, 8192, 512)
    data = oracle.make_inputs(shape, 11, "uniform")
    _check(_run(data, 1), oracle.reference_forward(*data))


def test_keys_matches_stream_family(cuda_lib):
    shape = (1, 64, 16, 8192, 2048)
    data = [t.cuda() for t in oracle.make_inputs(shape, 3, "normal")]
    a = dsa_b200.forward(*data, config=dsa_b200.Tuning(16, 32, 1))
    b = dsa_b200.forward(*data, config=_tuning(1))
    torch.cuda.synchronize()
    m = oracle.accuracy([t.float().cpu() for t in b], [t.float().cpu() for t in a])
    assert m["output"]["max_normalized"] < 5e-3 and m["maximum"]["max_normalized"] < 1e-6, m


@pytest.mark.parametrize("name,variant,split", [("decode_tp8", "uniform", 2), ("decode_tp8", "duplicates", 2),
                                                ("prefill_tp8", "uniform", 1)])
def test_keys_benchmark_configs(cuda_lib, name, variant, split):
    shape = bench.CONFIGS[name]
    data = bench.make_device_inputs(shape, bench.SEED, variant, "cuda")
    out, mx, sm = dsa_b200.forward(*data, config=_tuning(split))
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    b, s, h, _, _ = shape
    assert bool(torch.isfinite(out.float()).all()) and bool((sm >= 1.0 - 1e-6).all())
    rows = list(range(b * s)) if b * s <= 64 else list(range(0, b * s, 37)) + [b * s - 1]
    ref = oracle.reference_forward(*bench.compact_for_oracle(data, rows))
    rows_t = torch.as_tensor(rows, device="cuda")
    got = (out.reshape(b * s, h, 512)[rows_t].unsqueeze(1),
           mx.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h),
           sm.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h))
    _check(got, ref)
