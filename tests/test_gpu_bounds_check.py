"""The bounds-checking debug build (libdsa_b200_checked.so, -DDSA_BOUNDS_CHECK).

Every kernel family runs small cases through the checked library: no check
may fire (status word 0) and the results must be bit-identical to the
regular build's (the checks only read indices and addresses). The checks
cover every gathered row index and batch row, every shared-memory stage
destination of a gather and the tensor-memory columns of the score and
output reads."""
import pytest
import torch

import dsa_b200
from dsa_b200 import _native
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu

CASES = [  # (shape, Tuning args or None, index family)
    ((1, 2, 128, 4096, 2048), None, "duplicates"),            # split-V, cluster merge
    ((1, 1, 128, 4096, 2048), (128, 32, 32, 256), "invalid"),  # split-V + merge kernel
    ((1, 80, 128, 4096, 256), (128, 32, 1, 512), "normal"),    # pair
    ((1, 64, 16, 1024, 256), (16, 32, 1, 128), "invalid"),     # union + pair
    ((4, 1, 16, 8192, 2048), (16, 32, 8, 512), "duplicates"),  # stream, cluster merge
    ((4, 1, 16, 8192, 2048), (16, 32, 16, 512), "invalid"),    # stream + merge kernel
    ((2, 2, 32, 4096, 512), (16, 64, 2, 128), "normal"),       # keys
    ((2, 2, 32, 4096, 512), (16, 64, 3, 512), "invalid"),      # warp-MMA + merge
]


@pytest.mark.parametrize("shape,tuning,family", CASES)
def test_checked_build_is_silent_and_identical(cuda_lib, shape, tuning, family):
    checked = _native.load_checked()
    data = [t.cuda() for t in oracle.make_inputs(shape, 20261103, family)]
    config = None if tuning is None else dsa_b200.Tuning(*tuning[:3], pv_cols=tuning[3])
    dsa_b200.clear_device_status()
    plan = dsa_b200.ForwardPlan(*data, config=config)
    ref = [t.clone() for t in plan.run()]
    plan._lib = checked
    got = plan.run()
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    assert all(torch.equal(a, b) for a, b in zip(ref, got))
