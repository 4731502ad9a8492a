"""dsa_sparse_mla_fwd_noalloc: the forward for callers that cannot allocate.

Some callers of this library may not call cudaMalloc on the forward path: a
serving engine whose memory pool already holds the GPU's HBM, code that must
not pay cudaFree's device-wide synchronisation, or an FFI host that only owns
the input and output buffers. For them the library keeps the split-KV
partials in its own fixed-size device array instead of a caller workspace.

This test calls the variant through the C ABI three times in a row, with
different shapes and launch entries (32- and 64-key tiles; each call runs over
the previous call's leftovers in the shared array), and checks each result against the regular
entry point with a workspace, within the parity tolerance of the GPU tests.
It also checks that a problem whose partials exceed the array is refused.
The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

from dsa_b200 import _native
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu


def _args(data, out, mx, sm, launch):
    a = _native.FwdArgs()
    a.q, a.kv, a.q_rope, a.k_rope, a.indices = [t.data_ptr() for t in data]
    a.output, a.softmax_max, a.softmax_sum = out.data_ptr(), mx.data_ptr(), sm.data_ptr()
    b, s, h, _ = data[0].shape
    a.batch, a.queries, a.heads = b, s, h
    a.length, a.topk = data[1].shape[1], data[4].shape[-1]
    a.launch = launch
    return a


def _outputs(data):
    b, s, h, _ = data[0].shape
    out = torch.empty_like(data[0])
    mx = torch.empty((b, 1, s, h), dtype=torch.float32, device="cuda")
    return out, mx, torch.empty_like(mx)


def _with_workspace(lib, data, launch):
    out, mx, sm = _outputs(data)
    a = _args(data, out, mx, sm, launch)
    ws = lib.dsa_fwd_workspace_bytes(ctypes.byref(a))
    buf = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = buf.data_ptr(), ws
    assert lib.dsa_sparse_mla_fwd(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    return out, mx, sm


def _no_alloc(lib, data, launch):
    out, mx, sm = _outputs(data)
    a = _args(data, out, mx, sm, launch)
    code = lib.dsa_sparse_mla_fwd_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert code == _native.STATUS_OK, _native.status_string(code)
    torch.cuda.synchronize()
    return out, mx, sm


def test_no_alloc_matches_workspace_entry_point(cuda_lib):
    cases = [
        ((2, 2, 64, 8192, 2048), 20261103, _native.Launch(_native.FAMILY_WARP_MMA, 16, 32, 6)),
        ((1, 3, 32, 4096, 512), 20261102, _native.Launch(_native.FAMILY_AUTO, 0, 0, 0)),
        ((1, 2, 32, 4096, 1024), 5, _native.Launch(_native.FAMILY_WARP_MMA, 16, 64, 4)),
    ]
    for shape, seed, launch in cases:  # calls in a row over the shared array
        data = [t.cuda() for t in oracle.make_inputs(shape, seed, "normal")]
        expected = _with_workspace(cuda_lib, data, launch)
        got = _no_alloc(cuda_lib, data, launch)
        metrics = oracle.accuracy([t.float().cpu() for t in got], [t.float().cpu() for t in expected])
        assert oracle.passes(metrics), metrics


def test_no_alloc_refuses_oversized_partials(cuda_lib):
    # The call is refused before any launch, so plain zero tensors suffice.
    b, s, h, length, k = 64, 1, 128, 64, 2048
    bf = dict(dtype=torch.bfloat16, device="cuda")
    data = [torch.zeros((b, s, h, 512), **bf), torch.zeros((b, length, 1, 512), **bf),
            torch.zeros((b, s, h, 64), **bf), torch.zeros((b, length, 1, 64), **bf),
            torch.zeros((b, s, 1, k), dtype=torch.int32, device="cuda")]
    out, mx, sm = _outputs(data)
    launch = _native.Launch(_native.FAMILY_WARP_MMA, 16, 32, 16)
    rows = 64 * 16 * 128
    assert rows * 2056 > _native.NOALLOC_SCRATCH_BYTES
    a = _args(data, out, mx, sm, launch)
    code = cuda_lib.dsa_sparse_mla_fwd_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert code == _native.STATUS_WORKSPACE_TOO_SMALL
