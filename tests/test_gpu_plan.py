"""ForwardPlan: prepared forward, equal to forward() and CUDA-graph capturable."""
import pytest
import torch

import dsa_b200
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(1, 2, 128, 4096, 192), (2, 3, 16, 4096, 256), (1, 160, 128, 8192, 256)])
def test_plan_matches_forward(cuda_lib, shape):
    data = [t.cuda() for t in oracle.make_inputs(shape, 7, "normal")]
    ref = dsa_b200.forward(*data)
    plan = dsa_b200.ForwardPlan(*data)
    got = plan.run()
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    for a, b in zip(got, ref):
        assert torch.equal(a, b)


def test_plan_graph_replay_tracks_inputs(cuda_lib):
    shape = (2, 4, 128, 4096, 512)
    data = [t.cuda() for t in oracle.make_inputs(shape, 8, "normal")]
    plan = dsa_b200.ForwardPlan(*data)
    plan.run()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        plan.run()
    # new values in place, same addresses: the replay must see them
    fresh = oracle.make_inputs(shape, 9, "peaked")
    for dst, src in zip(data, fresh):
        dst.copy_(src)
    graph.replay()
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    metrics = oracle.accuracy([t.float().cpu() for t in plan.outputs], oracle.reference_forward(*fresh))
    assert oracle.passes(metrics), metrics
    del graph
