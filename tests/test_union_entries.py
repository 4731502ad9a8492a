"""The union launch's decomposition, checked on the CPU.

The union launch (family 6) runs 128 / H consecutive queries of one batch
row as one 128-row query over the union of their selected keys. For each
block it builds, in ascending key order, one entry per (key, repeat): the
key in bits 0-23 and one membership bit per query in bits 24-31, entry e of
a key holding the queries that selected the key more than e times; a block
without a valid index gets one entry that no query selects. Each softmax
row then takes the keys whose entry carries its query's bit.

This test restates that construction and shows, in float64, that attention
over the entries reproduces every query's attention over its own indices,
with duplicates keeping their repeated weight and invalid indices masked
(dsa/workspace.py:242-318, checked against the oracle with the benchmark
gates), that the entry count stays within the workspace cap of
(queries per block) x TOPK, and that no entry equals -1, the value the
kernel reads as "no index".
"""
import numpy as np
import pytest
import torch

from oracle import sparse_mla as oracle


def union_entries(block_ids, length):
    """Entries of one block: block_ids is [qpb, topk] int, returns int32 [n]."""
    qpb = block_ids.shape[0]
    counts = np.zeros((length, qpb), dtype=np.int64)
    for q in range(qpb):
        ids = block_ids[q]
        ids = ids[(ids >= 0) & (ids < length)]
        np.add.at(counts[:, q], ids, 1)
    entries = []
    for key in np.nonzero(counts.max(axis=1))[0]:
        for e in range(int(counts[key].max())):
            bits = sum(1 << q for q in range(qpb) if counts[key, q] > e)
            entries.append(int(key) | (bits << 24))
    if not entries:
        entries = [0]
    return np.array(entries, dtype=np.int64).astype(np.uint32).view(np.int32)


def attention_over_entries(q, q_rope, kv, k_rope, entries, query):
    """Float64 attention of one query's head rows over the entries with its bit."""
    raw = entries.view(np.uint32).astype(np.int64)
    keys = raw[((raw >> (24 + query)) & 1) == 1] & 0xFFFFFF
    heads = q.shape[0]
    if keys.size == 0:
        return torch.zeros(heads, 512, dtype=torch.float64), torch.full((heads,), -float("inf"), dtype=torch.float64), \
            torch.zeros(heads, dtype=torch.float64)
    keys = torch.as_tensor(keys)
    sel, rope = kv[keys].double(), k_rope[keys].double()
    score = (q.double() @ sel.T + q_rope.double() @ rope.T) / 24.0
    maximum = score.amax(-1)
    p = (score - maximum[:, None]).exp()
    total = p.sum(-1)
    return (p / total[:, None]) @ sel, maximum, total


@pytest.mark.parametrize("heads", [16, 32, 64])
@pytest.mark.parametrize("family", ["normal", "duplicates", "invalid"])
def test_union_entries_reproduce_per_query_attention(heads, family):
    qpb = 128 // heads
    shape = (1, 2 * qpb, heads, 300, 64)
    q, kv, qr, kr, idx = oracle.make_inputs(shape, 17, family)
    ref_out, ref_max, ref_sum = oracle.reference_forward(q, kv, qr, kr, idx)
    ids = idx[0, :, 0].numpy()
    outs, maxs, sums = [], [], []
    for b0 in range(0, shape[1], qpb):
        entries = union_entries(ids[b0:b0 + qpb], shape[3])
        assert entries.size <= qpb * shape[4]
        assert not (entries == -1).any()
        for j in range(qpb):
            o, m, s = attention_over_entries(q[0, b0 + j], qr[0, b0 + j], kv[0, :, 0], kr[0, :, 0], entries, j)
            outs.append(o)
            maxs.append(m)
            sums.append(s)
    got = (torch.stack(outs).unsqueeze(0), torch.stack(maxs).unsqueeze(0).unsqueeze(0),
           torch.stack(sums).unsqueeze(0).unsqueeze(0))
    metrics = oracle.accuracy([t.float() for t in got], [ref_out, ref_max, ref_sum])
    assert oracle.passes(metrics), metrics


def test_union_entries_repeat_counts():
    """A key chosen twice by one query and once by another: two entries, the
    first with both bits, the second with the first query's bit only."""
    ids = np.array([[5, 5, 7], [5, 9, -1]])
    entries = union_entries(ids, 10).view(np.uint32).astype(np.int64)
    assert [(int(e) & 0xFFFFFF, int(e) >> 24) for e in entries] == [(5, 0b11), (5, 0b01), (7, 0b01), (9, 0b10)]


def test_union_entries_block_without_valid_index():
    entries = union_entries(np.array([[-1, 12], [-3, 40]]), 10)
    assert entries.tolist() == [0]  # one entry that no query selects
