"""GPU parity: dsa_b200.forward (sm_100a library) against the CPU oracle.

Gates (oracle.GATES): output max-normalised error <= 5e-3 (the reference's
gate, tools/review.py:171); softmax_max and softmax_sum max-normalised error
<= 1e-5 (the benchmark contract). Index handling is exact: duplicates keep
their weight, invalid indices are masked, ragged TOPK tails are handled.
"""
import ctypes

import pytest
import torch

import bench
import dsa_b200
from dsa_b200 import _native
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu


def _gpu(data):
    return [t.cuda() for t in data]


def _check(got, ref, gates=oracle.GATES):
    metrics = oracle.accuracy([t.float().cpu() for t in got], ref)
    assert oracle.passes(metrics, gates), metrics
    return metrics


def test_library_loaded(cuda_lib):
    assert cuda_lib.dsa_abi_version() == _native.ABI_VERSION


@pytest.mark.parametrize("heads", [16, 32, 64, 128])
@pytest.mark.parametrize("family", oracle.FAMILIES)
def test_families_small(cuda_lib, heads, family):
    shape = (2, 3, heads, 4096, 256)
    data = oracle.make_inputs(shape, 20261103, family)
    out = dsa_b200.forward(*_gpu(data))
    torch.cuda.synchronize()
    _check(out, oracle.reference_forward(*data))


@pytest.mark.parametrize("topk", [1, 7, 31, 32, 33, 100, 2048, 2049])
def test_topk_tails(cuda_lib, topk):
    shape = (1, 2, 32, 3000, topk)
    data = oracle.make_inputs(shape, 5, "normal")
    out = dsa_b200.forward(*_gpu(data))
    torch.cuda.synchronize()
    _check(out, oracle.reference_forward(*data))


@pytest.mark.parametrize("bn", [32, 64])
@pytest.mark.parametrize("split", [1, 2, 3, 7, 16])
def test_explicit_splits(cuda_lib, bn, split):
    shape = (1, 2, 64, 8192, 2048)
    data = oracle.make_inputs(shape, 20261102, "peaked")
    out, kernels = dsa_b200.forward(*_gpu(data), config=dsa_b200.Tuning(16, bn, split), return_kernels=True)
    torch.cuda.synchronize()
    # the stream family (bn 32) merges splits 2..8 in its cluster launch
    merged_in_kernel = split == 1 or (bn == 32 and split <= 8)
    assert [k.name for k in kernels][-1:] == (["dsa_fwd_stream"] if bn == 32 and merged_in_kernel else
                                             ["dsa_merge"] if split > 1 else ["dsa_fwd_warp_mma"])
    assert len(kernels) == (1 if merged_in_kernel else 2)
    _check(out, oracle.reference_forward(*data))


@pytest.mark.parametrize("topk", [64, 80])
def test_stream_items_per_cta(cuda_lib, topk):
    """The persistent stream launch (split 1) with more items than resident
    CTAs: each CTA runs several items, and its gather ring carries on from
    one item's last tile into the next item's first (odd tile counts too)."""
    shape = (1, 700, 16, 2048, topk)
    data = oracle.make_inputs(shape, 11, "normal")
    out, kernels = dsa_b200.forward(*_gpu(data), config=dsa_b200.Tuning(16, 32, 1), return_kernels=True)
    torch.cuda.synchronize()
    assert [k.name for k in kernels] == ["dsa_fwd_stream"], kernels
    _check(out, oracle.reference_forward(*data))


def test_invalid_and_duplicate_index_semantics(cuda_lib):
    shape = (1, 1, 16, 256, 8)
    q, kv, qr, kr, _ = oracle.make_inputs(shape, 7, "normal")
    cases = [[5, 5, 9, -1, 256, 300, -7, 9], [0, 255, 255, 255, -1, -1, -1, 1]]
    for row in cases:
        ids = torch.tensor(row, dtype=torch.int32).reshape(1, 1, 1, 8)
        data = (q, kv, qr, kr, ids)
        out = dsa_b200.forward(*_gpu(data))
        torch.cuda.synchronize()
        _check(out, oracle.reference_forward(*data))


PIN_CASES = ["decode_b1", "decode_b8", "decode_tp8", "decode_b4_h16", "decode_b4_h32", "decode_b4_h64",
             "decode_b4_h128", "prefill_q16", "prefill_tp8", "prefill_k512", "decode_b32", "prefill_q64"]


@pytest.mark.parametrize("case", PIN_CASES)
def test_reference_shapes(cuda_lib, case):
    shape = dsa_b200.CASE_SHAPES[case]
    data = oracle.make_inputs(shape, 20261102, "normal")
    out = dsa_b200.forward(*_gpu(data))
    torch.cuda.synchronize()
    _check(out, oracle.reference_forward(*data))


@pytest.mark.parametrize("family", ["duplicates", "invalid"])
@pytest.mark.parametrize("case", ["decode_b1", "decode_b8"])
def test_reference_public_families(cuda_lib, case, family):
    shape = dsa_b200.CASE_SHAPES[case]
    data = oracle.make_inputs(shape, 20261103, family)
    out = dsa_b200.forward(*_gpu(data))
    torch.cuda.synchronize()
    _check(out, oracle.reference_forward(*data))


def _bench_parity(name, variant, sample_rows):
    shape = bench.CONFIGS[name]
    data = bench.make_device_inputs(shape, bench.SEED, variant, "cuda")
    out, mx, sm = dsa_b200.forward(*data)
    torch.cuda.synchronize()
    b, s, h, _, _ = shape
    # full-size properties: finite; the max term contributes exp(0) = 1
    assert bool(torch.isfinite(out.float()).all())
    assert bool(torch.isfinite(mx).all()) and bool((sm >= 1.0 - 1e-6).all())
    assert bool((sm <= shape[4] + 1e-3).all())
    rows = sample_rows if sample_rows is not None else list(range(b * s))
    ref = oracle.reference_forward(*bench.compact_for_oracle(data, rows))
    rows_t = torch.as_tensor(rows, device="cuda")
    got = (out.reshape(b * s, h, 512)[rows_t].unsqueeze(1), mx.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h),
           sm.reshape(b * s, h)[rows_t].reshape(len(rows), 1, 1, h))
    return _check(got, ref)


@pytest.mark.parametrize("name,variant,rows", [
    ("decode_b1", "uniform", None),
    ("decode_b8", "uniform", None),
    ("decode_tp8", "uniform", None),
    ("decode_tp8", "peaked", None),
    ("decode_tp8", "duplicates", None),
    ("prefill_tp8", "uniform", list(range(0, 4096, 7))),
    ("prefill_h128", "uniform", list(range(0, 16384, 257)) + [16383]),
])
def test_benchmark_configs(cuda_lib, name, variant, rows):
    _bench_parity(name, variant, rows)


def test_split_invariance_full_size(cuda_lib):
    """A size-independent property at a full benchmark size: the split-KV
    path (partials + FP32 merge) and the unsplit path agree."""
    shape = bench.CONFIGS["decode_tp8"]
    data = bench.make_device_inputs(shape, bench.SEED, "uniform", "cuda")
    a = dsa_b200.forward(*data, config=dsa_b200.Tuning(16, 32, 1))
    b = dsa_b200.forward(*data, config=dsa_b200.Tuning(16, 32, 8))
    torch.cuda.synchronize()
    m = oracle.accuracy([t.float().cpu() for t in b], [t.float().cpu() for t in a])
    assert m["output"]["max_normalized"] < 5e-3, m
    assert m["maximum"]["max_normalized"] == 0.0, m
    assert m["denominator"]["max_normalized"] < 1e-5, m


@pytest.mark.parametrize("s", [1, 4, 5, 16, 17, 40])  # warp-per-row kernel up to 16 splits, block kernel above
def test_merge_entry_point(cuda_lib, s):
    t, h = 5, 32
    g = torch.Generator().manual_seed(1)
    num = torch.randn((t, s, h, 512), generator=g)
    pm = torch.randn((t, s, h), generator=g) * 3
    pl = torch.rand((t, s, h), generator=g) * 50 + 1
    if s > 2:
        pm[1, 2] = oracle.FLT_MAX * -1  # an all-masked split merges with weight 0
        pl[1, 2] = 0
        num[1, 2] = 0
    ref = oracle.merge_partials(num, pm, pl)
    dn, dm, dl = num.cuda(), pm.cuda(), pl.cuda()
    out = torch.empty((t, h, 512), dtype=torch.bfloat16, device="cuda")
    om = torch.empty((t, h), device="cuda")
    ol = torch.empty((t, h), device="cuda")
    code = cuda_lib.dsa_merge_partials(dn.data_ptr(), dm.data_ptr(), dl.data_ptr(), out.data_ptr(),
                                       om.data_ptr(), ol.data_ptr(), t, h, s,
                                       torch.cuda.current_stream().cuda_stream)
    assert code == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ref[0], rtol=8e-3, atol=1e-6)
    torch.testing.assert_close(om.cpu(), ref[1], rtol=0, atol=0)
    torch.testing.assert_close(ol.cpu(), ref[2], rtol=2e-6, atol=1e-6)


def test_c_abi_direct_call_matches_api(cuda_lib):
    shape = (2, 2, 32, 1024, 128)
    data = _gpu(oracle.make_inputs(shape, 9, "normal"))
    ref = dsa_b200.forward(*data)
    out = torch.empty_like(data[0])
    mx = torch.empty((2, 1, 2, 32), device="cuda")
    sm = torch.empty_like(mx)
    args = _native.FwdArgs()
    args.q, args.kv, args.q_rope, args.k_rope, args.indices = [t.data_ptr() for t in data]
    args.output, args.softmax_max, args.softmax_sum = out.data_ptr(), mx.data_ptr(), sm.data_ptr()
    args.batch, args.queries, args.heads, args.length, args.topk = shape
    args.launch = _native.Launch(0, 0, 0, 0)
    ws = cuda_lib.dsa_fwd_workspace_bytes(ctypes.byref(args))
    buf = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
    args.workspace, args.workspace_bytes = buf.data_ptr(), ws
    assert cuda_lib.dsa_sparse_mla_fwd(ctypes.byref(args), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, ref[0]) and torch.equal(mx, ref[1]) and torch.equal(sm, ref[2])


def _abi_forward(cuda_lib, data, shape, launch, out_offset):
    """One call through the C ABI with the output starting `out_offset`
    BF16 elements into its buffer."""
    b, s, h, _, _ = shape
    buf = torch.empty(b * s * h * 512 + out_offset, dtype=torch.bfloat16, device="cuda")
    out = buf[out_offset:].view(b, s, h, 512)
    mx = torch.empty((b, 1, s, h), device="cuda")
    sm = torch.empty_like(mx)
    args = _native.FwdArgs()
    args.q, args.kv, args.q_rope, args.k_rope, args.indices = [t.data_ptr() for t in data]
    args.output, args.softmax_max, args.softmax_sum = out.data_ptr(), mx.data_ptr(), sm.data_ptr()
    args.batch, args.queries, args.heads, args.length, args.topk = shape
    args.launch = launch
    ws = cuda_lib.dsa_fwd_workspace_bytes(ctypes.byref(args))
    wbuf = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
    args.workspace, args.workspace_bytes = wbuf.data_ptr(), ws
    assert cuda_lib.dsa_sparse_mla_fwd(ctypes.byref(args), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    return out.clone(), mx, sm


@pytest.mark.parametrize("shape,launch", [
    ((1, 80, 128, 4096, 256), (_native.FAMILY_UMMA_PAIR, 128, 32, 1)),   # pair, paired row stores
    ((1, 2, 128, 4096, 256), (_native.FAMILY_UMMA, 128, 32, 1)),          # split-V, row stores
    ((2, 1, 128, 4096, 512), (_native.FAMILY_UMMA, 128, 32, 4)),          # split-V, merge in the cluster
    ((1, 64, 16, 1024, 256), (_native.FAMILY_PAIR_UNION, 128, 32, 1)),    # union launch
    ((2, 3, 16, 4096, 256), (_native.FAMILY_STREAM, 16, 32, 1)),
    ((2, 1, 16, 4096, 1024), (_native.FAMILY_STREAM, 16, 32, 4)),        # stream, merge in the cluster
    ((2, 3, 16, 4096, 256), (_native.FAMILY_WARP_MMA, 16, 32, 1)),
], ids=["pair", "split-V", "split-V-cluster", "union", "stream", "stream-cluster", "warp-MMA"])
def test_output_16_byte_aligned(cuda_lib, shape, launch):
    """The C ABI accepts an output that is 16- but not 32-byte aligned: the
    families then take their 16-byte store paths, with bit-identical
    results."""
    data = _gpu(oracle.make_inputs(shape, 13, "normal"))
    la = _native.Launch(*launch)
    aligned = _abi_forward(cuda_lib, data, shape, la, 0)
    offset = _abi_forward(cuda_lib, data, shape, la, 8)  # 16 bytes into a 512-byte aligned buffer
    for x, y in zip(aligned, offset):
        assert torch.equal(x, y)
    _check(offset, oracle.reference_forward(*[t.cpu() for t in data]))


def test_workspace_too_small_is_reported(cuda_lib):
    shape = (1, 1, 32, 1024, 256)
    data = _gpu(oracle.make_inputs(shape, 9, "normal"))
    args = _native.FwdArgs()
    args.q, args.kv, args.q_rope, args.k_rope, args.indices = [t.data_ptr() for t in data]
    out = torch.empty_like(data[0])
    mx = torch.empty((1, 1, 1, 32), device="cuda")
    args.output, args.softmax_max, args.softmax_sum = out.data_ptr(), mx.data_ptr(), mx.data_ptr()
    args.batch, args.queries, args.heads, args.length, args.topk = shape
    args.launch = _native.Launch(1, 16, 32, 4)
    assert cuda_lib.dsa_sparse_mla_fwd(ctypes.byref(args), None) == _native.STATUS_WORKSPACE_TOO_SMALL


def test_inputs_not_modified_and_deterministic(cuda_lib):
    shape = (1, 4, 64, 2048, 512)
    data = _gpu(oracle.make_inputs(shape, 13, "duplicates"))
    before = [t.clone() for t in data]
    a = dsa_b200.forward(*data)
    b = dsa_b200.forward(*data)
    torch.cuda.synchronize()
    for x, y in zip(before, data):
        assert torch.equal(x, y)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    assert dsa_b200.device_status() == 0
