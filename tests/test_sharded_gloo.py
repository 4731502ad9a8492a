"""Query-sharding and output gather on CPU ranks (gloo, world_size 2 and 3).

The per-rank compute is the CPU oracle (test-only stand-in for the GPU
forward); what is checked is the partition into contiguous pieces and the
all-gather that reassembles the full outputs.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsa_b200 import sharded


def test_shard_bounds_cover_exactly():
    for total in (1, 7, 16, 16384, 4097):
        for world in (1, 2, 3, 4, 8):
            rows = []
            for r in range(world):
                lo, hi = sharded.shard_bounds(total, world, r)
                rows.extend(range(lo, hi))
            assert rows == list(range(total))


def test_pieces_are_contiguous_views():
    for queries in (1, 5, 4096):
        for lo, hi in ((0, queries * 3), (2, queries * 2 + 1), (queries, queries + 1)):
            if hi <= lo:
                continue
            pieces = sharded.shard_pieces(queries, lo, hi)
            rows = []
            for b0, b1, s0, s1 in pieces:
                assert b1 > b0 and s1 > s0
                assert b1 - b0 == 1 or (s0 == 0 and s1 == queries)
                rows.extend(b * queries + s for b in range(b0, b1) for s in range(s0, s1))
            assert rows == list(range(lo, hi))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_fn(q, kv, qr, kr, ids):
    from oracle import sparse_mla as oracle
    out, mx, sm = oracle.reference_forward(q, kv, qr, kr, ids)
    return out, mx, sm


def _worker(rank, world, port, shape, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import sparse_mla as oracle
        data = oracle.make_inputs(shape, 99, "normal")
        out, mx, sm = sharded.sharded_forward(*data, fn=_oracle_fn)
        full = oracle.reference_forward(*data)
        ok = (torch.equal(out, full[0]) and torch.equal(mx, full[1]) and torch.equal(sm, full[2]))
        queue.put((rank, ok, tuple(out.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,shape", [(2, (2, 3, 16, 256, 32)), (3, (1, 7, 16, 128, 16))])
def test_sharded_forward_gloo(world, shape):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, out_shape in results:
        assert ok, rank
        assert out_shape == (shape[0], shape[1], shape[2], 512)
