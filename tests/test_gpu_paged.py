"""GPU parity of the paged KV cache forward against the oracle's dense
restatement, and bit-identity with the dense forward on the same logical
data (same kernels, same key order)."""
import pytest
import torch

import dsa_b200
from oracle import sparse_mla as oracle
from test_paged import make_pool

pytestmark = pytest.mark.gpu


def _check(got, ref):
    metrics = oracle.accuracy([t.float().cpu() for t in got], ref)
    assert oracle.passes(metrics), metrics


@pytest.mark.parametrize("heads", [16, 128])
def test_paged_matches_oracle(cuda_lib, heads):
    batch, queries, max_blocks, block_size, num_blocks, topk = 2, 3, 32, 64, 80, 512
    kv, kr, kv_cache, kr_cache, table = make_pool(batch, max_blocks, block_size, num_blocks, 7)
    g = torch.Generator().manual_seed(9)
    q = torch.randn((batch, queries, heads, 512), generator=g).bfloat16()
    qr = torch.randn((batch, queries, heads, 64), generator=g).bfloat16()
    ids = torch.stack([torch.randperm(2100, generator=g)[:topk] for _ in range(batch * queries)]).int()
    ids = ids.reshape(batch, queries, 1, topk)
    ids[0, 1, 0, :7] = -1
    seq = torch.tensor([2000, 1500], dtype=torch.int32)
    table[1, 30] = -1  # a hole in the table: those tokens are masked
    out = dsa_b200.forward_paged(*[t.cuda() for t in (q, kv_cache, qr, kr_cache, table, ids)],
                                 seq_lens=seq.cuda())
    torch.cuda.synchronize()
    assert dsa_b200.device_status() == 0
    dkv, dkr, dids = oracle.paged_to_dense(kv_cache, kr_cache, table, ids, seq)
    _check(out, oracle.reference_forward(q, dkv, qr, dkr, dids))


@pytest.mark.parametrize("queries", [2, 80])  # split-V and pair families
def test_paged_is_bit_identical_to_dense(cuda_lib, queries):
    batch, max_blocks, block_size, num_blocks, topk = 1, 16, 128, 40, 1024
    kv, kr, kv_cache, kr_cache, table = make_pool(batch, max_blocks, block_size, num_blocks, 11)
    g = torch.Generator().manual_seed(5)
    q = torch.randn((batch, queries, 128, 512), generator=g).bfloat16()
    qr = torch.randn((batch, queries, 128, 64), generator=g).bfloat16()
    length = max_blocks * block_size
    ids = torch.stack([torch.randperm(length, generator=g)[:topk] for _ in range(batch * queries)]).int()
    ids = ids.reshape(batch, queries, 1, topk)
    dense = dsa_b200.forward(*[t.cuda() for t in (q, kv, qr, kr, ids)])
    paged = dsa_b200.forward_paged(*[t.cuda() for t in (q, kv_cache, qr, kr_cache, table, ids)])
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(dense, paged))
