"""Paged KV cache (the KV-cache format the reference leaves out,
README.md:19-20): CPU checks of the oracle restatement, the argument rules
and the workspace query; the GPU parity tests are in test_gpu_paged.py."""
import ctypes

import pytest
import torch

import dsa_b200
from dsa_b200 import _native, api
from oracle import sparse_mla as oracle


def make_pool(batch, max_blocks, block_size, num_blocks, seed):
    """A dense logical cache scattered into a shuffled page pool."""
    g = torch.Generator().manual_seed(seed)
    kv = torch.randn((batch, max_blocks * block_size, 1, 512), generator=g).bfloat16()
    kr = torch.randn((batch, max_blocks * block_size, 1, 64), generator=g).bfloat16()
    perm = torch.randperm(num_blocks, generator=g)[:batch * max_blocks].reshape(batch, max_blocks).int()
    kv_cache = torch.randn((num_blocks, block_size, 1, 512), generator=g).bfloat16()
    kr_cache = torch.randn((num_blocks, block_size, 1, 64), generator=g).bfloat16()
    for b in range(batch):
        for j in range(max_blocks):
            kv_cache[perm[b, j]] = kv[b, j * block_size:(j + 1) * block_size]
            kr_cache[perm[b, j]] = kr[b, j * block_size:(j + 1) * block_size]
    return kv, kr, kv_cache, kr_cache, perm


def test_paged_to_dense_restatement():
    kv, kr, kv_cache, kr_cache, table = make_pool(2, 4, 16, 11, 3)
    ids = torch.tensor([0, 5, 17, 63, 64, -1, 40, 47], dtype=torch.int32).reshape(1, 1, 1, 8).repeat(2, 1, 1, 1)
    seq = torch.tensor([64, 41], dtype=torch.int32)
    table_bad = table.clone()
    table_bad[1, 2] = -1  # tokens 32..47 of row 1 have no block
    dkv, dkr, dids = oracle.paged_to_dense(kv_cache, kr_cache, table_bad, ids, seq)
    assert torch.equal(dkv[0], kv[0]) and torch.equal(dkr[0], kr[0])
    assert torch.equal(dkv[1, :32], kv[1, :32]) and torch.equal(dkv[1, 48:], kv[1, 48:])
    assert torch.equal(dids[0, 0, 0], torch.tensor([0, 5, 17, 63, -1, -1, 40, 47], dtype=torch.int32))
    assert torch.equal(dids[1, 0, 0], torch.tensor([0, 5, 17, -1, -1, -1, -1, -1], dtype=torch.int32))


def test_paged_argument_rules(monkeypatch):
    monkeypatch.setattr(api, "DEVICE_TYPE", "meta")
    m = dict(device="meta")
    q = torch.empty((2, 3, 128, 512), dtype=torch.bfloat16, **m)
    qr = torch.empty((2, 3, 128, 64), dtype=torch.bfloat16, **m)
    kvc = torch.empty((10, 64, 1, 512), dtype=torch.bfloat16, **m)
    krc = torch.empty((10, 64, 1, 64), dtype=torch.bfloat16, **m)
    table = torch.empty((2, 4), dtype=torch.int32, **m)
    ids = torch.empty((2, 3, 1, 128), dtype=torch.int32, **m)
    bad = [
        (q, kvc, qr, krc, table[:1], ids),                                        # table rows != B
        (q, kvc, qr, krc[:, :32], table, ids),                                     # rope pool shape
        (q, kvc.float(), qr, krc, table, ids),                                     # dtype
        (q, kvc, qr, krc, table.long(), ids),                                      # table dtype
    ]
    for args in bad:
        with pytest.raises(ValueError):
            dsa_b200.forward_paged(*args)
    with pytest.raises(ValueError):
        dsa_b200.forward_paged(q, kvc, qr, krc, table, ids, seq_lens=torch.empty((3,), dtype=torch.int32, **m))


def test_paged_workspace_bytes():
    lib = _native.load()
    a = _native.FwdArgs()
    a.batch, a.queries, a.heads, a.topk = 2, 3, 32, 256
    a.launch = _native.Launch(1, 16, 32, 4)
    pg = _native.PagedKv(1, None, 4, 64, 10)  # any non-null table pointer: no device access here
    ws = lib.dsa_fwd_paged_workspace_bytes(ctypes.byref(a), ctypes.byref(pg))
    rows = 2 * 3 * 4 * 32
    assert ws >= 2 * 3 * 256 * 4 + rows * 514 * 4 and ws % 256 == 0
    pg.block_size = 0
    assert lib.dsa_fwd_paged_workspace_bytes(ctypes.byref(a), ctypes.byref(pg)) == 0
