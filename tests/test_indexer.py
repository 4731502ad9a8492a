"""Lightning indexer + top-k (the stage the reference leaves out,
README.md:19-20): CPU checks of the oracle's tie rule, the argument rules and
the workspace query; GPU parity is in test_gpu_indexer.py."""
import ctypes

import pytest
import torch

import dsa_b200
from dsa_b200 import _native, api, indexer
from oracle import sparse_mla as oracle


def test_oracle_topk_tie_rule_and_padding():
    scores = torch.tensor([[[1.0, 3.0, 3.0, 2.0, 3.0, 0.5]]])
    assert oracle.topk_indices(scores, 2).flatten().tolist() == [1, 2]          # ties: smaller keys first
    assert oracle.topk_indices(scores, 4).flatten().tolist() == [1, 2, 3, 4]    # ascending key order
    lens = torch.tensor([[3]], dtype=torch.int32)
    assert oracle.topk_indices(scores, 4, lens).flatten().tolist() == [0, 1, 2, -1]


def test_oracle_scores_formula():
    q = torch.tensor([[[[1.0, 0.0], [0.0, 1.0]]]])          # B=1, SQ=1, HI=2, d=2
    k = torch.tensor([[[2.0, -1.0], [-3.0, 4.0]]])          # L=2
    w = torch.tensor([[[0.5, 2.0]]])
    s = oracle.indexer_scores(q, k, w)
    assert s.flatten().tolist() == [0.5 * 2.0 + 2.0 * 0.0, 0.5 * 0.0 + 2.0 * 4.0]


def test_indexer_workspace_bytes():
    lib = _native.load()
    a = _native.IndexerArgs()
    a.batch, a.queries, a.heads, a.length, a.topk = 2, 3, 64, 1000, 128
    assert lib.dsa_indexer_workspace_bytes(ctypes.byref(a)) >= 2 * 3 * 1000 * 4
    a.heads = 48
    assert lib.dsa_indexer_workspace_bytes(ctypes.byref(a)) == 0


def test_indexer_argument_rules(monkeypatch):
    monkeypatch.setattr(indexer, "DEVICE_TYPE", "meta")
    m = dict(device="meta")
    q = torch.empty((2, 3, 64, 128), dtype=torch.bfloat16, **m)
    k = torch.empty((2, 100, 128), dtype=torch.bfloat16, **m)
    w = torch.empty((2, 3, 64), dtype=torch.float32, **m)
    for args in [(q[..., :64], k, w, 8), (q, k[:1], w, 8), (q, k, w.double(), 8), (q, k, w, 0),
                 (q[:, :, :48], k, w[:, :, :48], 8)]:
        with pytest.raises(ValueError):
            dsa_b200.indexer_topk(*args)
