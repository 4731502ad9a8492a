"""GPU parity of the lightning indexer + top-k against the oracle
(oracle.indexer_scores / oracle.topk_indices). With small-integer inputs and
power-of-two weights every product and sum is exact in FP32, so scores and
indices must match exactly, ties included; random inputs are checked to FP32
rounding, and indices away from the selection threshold exactly."""
import pytest
import torch

import dsa_b200
from oracle import sparse_mla as oracle

pytestmark = pytest.mark.gpu


def _integer_case(batch, queries, heads, length, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-2, 3, (batch, queries, heads, 128), generator=g).bfloat16()
    k = torch.randint(-2, 3, (batch, length, 128), generator=g).bfloat16()
    w = 2.0 ** torch.randint(-2, 2, (batch, queries, heads), generator=g).float()
    return q, k, w


@pytest.mark.parametrize("heads", [16, 32, 64, 128])
@pytest.mark.parametrize("length,topk", [(1000, 100), (300, 2048), (4096, 2048)])
def test_indexer_exact(cuda_lib, heads, length, topk):
    q, k, w = _integer_case(2, 5, heads, length, heads + length)
    idx, sc = dsa_b200.indexer_topk(q.cuda(), k.cuda(), w.cuda(), topk, return_scores=True)
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    ref = oracle.indexer_scores(q, k, w)
    assert torch.equal(sc.cpu(), ref)
    assert torch.equal(idx.cpu(), oracle.topk_indices(ref, topk))


def test_indexer_lengths(cuda_lib):
    q, k, w = _integer_case(2, 6, 64, 2500, 3)
    lens = torch.tensor([[0, 1, 100, 1500, 2500, 9999], [2048, 2049, 7, 2000, 129, 128]], dtype=torch.int32)
    idx = dsa_b200.indexer_topk(q.cuda(), k.cuda(), w.cuda(), 2048, lengths=lens.cuda())
    torch.cuda.synchronize()
    assert torch.equal(idx.cpu(), oracle.topk_indices(oracle.indexer_scores(q, k, w), 2048, lens))


def test_indexer_random(cuda_lib):
    g = torch.Generator().manual_seed(20261103)
    b, s, h, length, topk = 2, 9, 64, 8192, 512
    q = torch.randn((b, s, h, 128), generator=g).bfloat16()
    k = torch.randn((b, length, 128), generator=g).bfloat16()
    w = torch.rand((b, s, h), generator=g) / h
    idx, sc = dsa_b200.indexer_topk(q.cuda(), k.cuda(), w.cuda(), topk, return_scores=True)
    torch.cuda.synchronize()
    ref = oracle.indexer_scores(q, k, w)
    sc = sc.cpu()
    tol = 1e-5 * ref.abs().amax(-1, keepdim=True)  # FP32 accumulation order
    assert bool(((sc - ref).abs() <= tol).all())
    # indices: exact wherever the oracle's score is not within the tolerance of the selection threshold
    got = idx.cpu()
    for bi in range(b):
        for si in range(s):
            thr = torch.sort(ref[bi, si], descending=True).values[topk - 1]
            near = (ref[bi, si] - thr).abs() <= 2 * tol[bi, si, 0]
            sel_got = torch.zeros(length, dtype=torch.bool)
            sel_got[got[bi, si, 0].long()] = True
            sel_ref = torch.zeros(length, dtype=torch.bool)
            sel_ref[oracle.topk_indices(ref[bi:bi + 1, si:si + 1], topk)[0, 0, 0].long()] = True
            assert bool(((sel_got == sel_ref) | near).all())
            assert bool((got[bi, si, 0, 1:] > got[bi, si, 0, :-1]).all())  # ascending, distinct


def test_indexer_feeds_forward(cuda_lib):
    """Indices from the indexer drive the sparse-MLA forward end to end."""
    b, s, h, length, topk = 1, 4, 128, 4096, 1024
    qi, ki, w = _integer_case(b, s, 64, length, 7)
    data = oracle.make_inputs((b, s, h, length, topk), 20261103, "normal")
    q, kv, qr, kr, _ = data
    idx = dsa_b200.indexer_topk(qi.cuda(), ki.cuda(), w.cuda(), topk)
    out = dsa_b200.forward(q.cuda(), kv.cuda(), qr.cuda(), kr.cuda(), idx)
    torch.cuda.synchronize()
    ref_idx = oracle.topk_indices(oracle.indexer_scores(qi, ki, w), topk)
    assert torch.equal(idx.cpu(), ref_idx)
    metrics = oracle.accuracy([t.float().cpu() for t in out], oracle.reference_forward(q, kv, qr, kr, ref_idx))
    assert oracle.passes(metrics), metrics


@pytest.mark.parametrize("budget_rows", [7, 1])  # pieces of whole batch rows / of queries in a row
def test_indexer_in_pieces(cuda_lib, monkeypatch, budget_rows):
    from dsa_b200 import indexer

    q, k, w = _integer_case(3, 8, 32, 1000, 11)
    monkeypatch.setattr(indexer, "SCORE_BUDGET", budget_rows * 1000 * 4)
    idx = dsa_b200.indexer_topk(q.cuda(), k.cuda(), w.cuda(), 64)
    torch.cuda.synchronize()
    assert torch.equal(idx.cpu(), oracle.topk_indices(oracle.indexer_scores(q, k, w), 64))
