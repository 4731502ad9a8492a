"""Device-side failure path: a bounded wait that runs out.

The reference bounds a hung run with a host-side watchdog
(tools/review.py:298-299). Here every device-side wait is bounded instead:
with ``dsa_set_wait_test`` the split-V family's first CTA waits on a barrier
that nothing arrives at, under a 1 ms bound. The wait runs out, the CTA sets
the timeout bit in the status word, waits for the tensor-core work it has
already issued, releases its tensor memory and leaves; the launch completes
and the context stays usable. Nothing here faults, traps or hangs a GPU:
every wait on this path is bounded.
"""
import time

import pytest
import torch

import dsa_b200
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu

SPLIT_V = dsa_b200.Tuning(128, 32, 4, pv_cols=256)
SHAPE = (1, 2, 128, 4096, 2048)


def test_bounded_wait_runs_out_and_is_reported(cuda_lib):
    data = oracle.make_inputs(SHAPE, 20261103, "normal")
    dev = [t.cuda() for t in data]
    dsa_b200.forward(*dev, config=SPLIT_V)  # first launch of the family outside the timing
    dsa_b200.clear_device_status()
    assert cuda_lib.dsa_set_wait_test(1_000_000, 1) == 0  # 1 ms bound; the first CTA stalls
    try:
        t0 = time.perf_counter()
        dsa_b200.forward(*dev, config=SPLIT_V)
        bits = dsa_b200.device_status()  # synchronises: the launch has completed
        elapsed = time.perf_counter() - t0
    finally:
        cuda_lib.dsa_set_wait_test(0, 0)
    assert bits & 1, bits
    # the runtime bound took effect: the built-in bound alone is 2 s
    assert elapsed < 1.0, elapsed
    with pytest.raises(RuntimeError, match="timed out"):
        dsa_b200.check_device_status()
    dsa_b200.clear_device_status()
    assert dsa_b200.device_status() == 0

    # the context is still usable: the same call without the stall passes parity
    out = dsa_b200.forward(*dev, config=SPLIT_V)
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    metrics = oracle.accuracy([t.float().cpu() for t in out], oracle.reference_forward(*data))
    assert oracle.passes(metrics), metrics


def test_runtime_bound_without_stall_changes_nothing(cuda_lib):
    """A short runtime bound that every wait meets leaves the result bit-identical."""
    dev = [t.cuda() for t in oracle.make_inputs(SHAPE, 3, "peaked")]
    dsa_b200.clear_device_status()
    ref = dsa_b200.forward(*dev, config=SPLIT_V)
    assert cuda_lib.dsa_set_wait_test(200_000_000, 0) == 0  # 200 ms
    try:
        got = dsa_b200.forward(*dev, config=SPLIT_V)
        torch.cuda.synchronize()
    finally:
        cuda_lib.dsa_set_wait_test(0, 0)
    assert dsa_b200.device_status() == 0
    assert all(torch.equal(a, b) for a, b in zip(ref, got))
