"""GPU parity of the two tcgen05/TMEM families (H = 128).

Selected explicitly with ``Tuning(bm=128, bn=32, split=S, pv_cols=C)``:
``pv_cols=256`` runs the split-V family (one CTA per half of the value
columns), ``pv_cols=512`` the pair family (score CTA + value CTA per
query). Both are checked against the CPU oracle with the same gates as the
generic family.
"""
import pytest
import torch

import bench
import dsa_b200
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[256, 512], ids=["splitv", "pair"])
def pv_cols(request):
    return request.param


def _run(data, split, pv_cols):
    out = dsa_b200.forward(*[t.cuda() for t in data], config=dsa_b200.Tuning(128, 32, split, pv_cols=pv_cols))
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0, "a bounded device-side wait timed out"
    return out


def _check(got, ref):
    got = [t.float().cpu() for t in got]
    metrics = oracle.accuracy(got, ref)
    if not oracle.passes(metrics):
        # locate the worst (token, head) of each statistic for the report
        where = {}
        for name, a, b in (("maximum", got[1], ref[1]), ("denominator", got[2], ref[2])):
            d = ((a - b).abs() / b.abs().max()).reshape(-1)
            k = int(d.argmax())
            where[name] = (k, float(a.reshape(-1)[k]), float(b.reshape(-1)[k]), float(d[k]))
        raise AssertionError(f"{metrics}\nworst (flat index, got, ref, err): {where}")
    return metrics


@pytest.mark.parametrize("split", [1, 2, 3])
def test_umma_small(cuda_lib, split, pv_cols):
    shape = (1, 2, 128, 4096, 192)
    data = oracle.make_inputs(shape, 20261103, "normal")
    _check(_run(data, split, pv_cols), oracle.reference_forward(*data))


@pytest.mark.parametrize("family", oracle.FAMILIES)
def test_umma_families(cuda_lib, family, pv_cols):
    shape = (2, 3, 128, 4096, 256)
    data = oracle.make_inputs(shape, 20261103, family)
    _check(_run(data, 1, pv_cols), oracle.reference_forward(*data))


@pytest.mark.parametrize("topk,split", [(1, 1), (31, 1), (32, 1), (33, 2), (100, 1), (2049, 5), (2048, 64)])
def test_umma_topk_tails(cuda_lib, topk, split, pv_cols):
    shape = (1, 2, 128, 3000, topk)
    data = oracle.make_inputs(shape, 5, "normal")
    _check(_run(data, split, pv_cols), oracle.reference_forward(*data))


@pytest.mark.parametrize("split", [1, 8, 32, 64])
def test_umma_reference_decode_b1(cuda_lib, split, pv_cols):
    shape = dsa_b200.CASE_SHAPES["decode_b1"]
    data = oracle.make_inputs(shape, 20261102, "normal")
    _check(_run(data, split, pv_cols), oracle.reference_forward(*data))


def test_umma_many_items_persistent(cuda_lib, pv_cols):
    """More work items than resident CTAs: every CTA loops over items."""
    shape = (2, 300, 128, 8192, 256)
    data = oracle.make_inputs(shape, 11, "peaked")
    _check(_run(data, 1, pv_cols), oracle.reference_forward(*data))


def test_umma_matches_generic_family(cuda_lib, pv_cols):
    shape = (1, 8, 128, 8192, 2048)
    data = [t.cuda() for t in oracle.make_inputs(shape, 3, "normal")]
    a = dsa_b200.forward(*data, config=dsa_b200.Tuning(16, 32, 1))
    b = dsa_b200.forward(*data, config=dsa_b200.Tuning(128, 32, 1, pv_cols=pv_cols))
    torch.cuda.synchronize()
    m = oracle.accuracy([t.float().cpu() for t in b], [t.float().cpu() for t in a])
    assert m["output"]["max_normalized"] < 5e-3 and m["maximum"]["max_normalized"] < 1e-6, m


@pytest.mark.parametrize("name,split", [("decode_b1", 32), ("decode_b8", 8), ("prefill_h128", 1)])
def test_umma_benchmark_configs(cuda_lib, name, split, pv_cols):
    shape = bench.CONFIGS[name]
    data = bench.make_device_inputs(shape, bench.SEED, "uniform", "cuda")
    out, mx, sm = dsa_b200.forward(*data, config=dsa_b200.Tuning(128, 32, split, pv_cols=pv_cols))
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    b, s, h, _, _ = shape
    assert bool(torch.isfinite(out.float()).all()) and bool((sm >= 1.0 - 1e-6).all())
    rows = list(range(b * s)) if b * s <= 64 else list(range(0, b * s, 263)) + [b * s - 1]
    ref = oracle.reference_forward(*bench.compact_for_oracle(data, rows))
    rows_t = torch.as_tensor(rows, device="cuda")
    got = (out.reshape(b * s, h, 512)[rows_t].unsqueeze(1),
           mx.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h),
           sm.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h))
    _check(got, ref)
