"""Query-sharded multi-GPU forward: one process per GPU, kv replicated.

Every (batch, query) row of the sparse-MLA forward is independent (the
reference's job grid already partitions on it, dsa/workspace.py:25-30), so
N ranks each take a contiguous range of the flattened B*SQ queries,
batch-major, run the single-GPU forward on it, and the only exchange is an
all-gather of the output and statistic shards afterwards. There is no
data-path collective inside the kernels.
"""
from __future__ import annotations

from typing import Callable, List, Tuple

import torch
import torch.distributed as dist


def shard_bounds(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, equal-width (last one possibly short) range of ``total``
    flattened queries owned by ``rank``."""
    per = -(-total // world)
    lo = min(rank * per, total)
    return lo, min(lo + per, total)


def shard_pieces(queries: int, lo: int, hi: int) -> List[Tuple[int, int, int, int]]:
    """Split flattened rows [lo, hi) into pieces ``(b0, b1, s0, s1)`` that each
    map to contiguous 4-D views ``x[b0:b1, s0:s1]`` (a partial batch row, or a
    run of whole batch rows)."""
    pieces = []
    row = lo
    while row < hi:
        b, s = divmod(row, queries)
        if s == 0 and hi - row >= queries:
            nb = (hi - row) // queries
            pieces.append((b, b + nb, 0, queries))
            row += nb * queries
        else:
            s1 = min(queries, s + (hi - row))
            pieces.append((b, b + 1, s, s1))
            row += s1 - s
    return pieces


def forward_pieces(q, kv, q_rope, k_rope, indices, lo, hi, fn: Callable):
    """Run ``fn`` (the single-device forward) on each piece of rows [lo, hi).
    Returns a list of ``(rows, (output, max, sum))``; no copies are made."""
    queries = q.shape[1]
    results = []
    for b0, b1, s0, s1 in shard_pieces(queries, lo, hi):
        res = fn(q[b0:b1, s0:s1], kv[b0:b1], q_rope[b0:b1, s0:s1], k_rope[b0:b1], indices[b0:b1, s0:s1])
        results.append(((b1 - b0) * (s1 - s0), res))
    return results


def assemble_local(results, heads, device, out_dtype=torch.bfloat16):
    """Concatenate piece results into flat local shards
    ``[rows, H, 512]``, ``[rows, H]``, ``[rows, H]``."""
    outs = [r[0].reshape(n, heads, 512) for n, r in results]
    mxs = [r[1].reshape(n, heads) for n, r in results]
    sms = [r[2].reshape(n, heads) for n, r in results]
    if len(outs) == 1:
        return outs[0], mxs[0], sms[0]
    if not outs:
        return (torch.empty((0, heads, 512), dtype=out_dtype, device=device),
                torch.empty((0, heads), dtype=torch.float32, device=device),
                torch.empty((0, heads), dtype=torch.float32, device=device))
    return torch.cat(outs), torch.cat(mxs), torch.cat(sms)


def _all_gather(flat: torch.Tensor, per: int, group) -> torch.Tensor:
    world = dist.get_world_size(group)
    shape = (per,) + tuple(flat.shape[1:])
    padded = flat
    if flat.shape[0] != per:
        padded = torch.zeros(shape, dtype=flat.dtype, device=flat.device)
        padded[:flat.shape[0]] = flat
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world * per,) + shape[1:], dtype=flat.dtype, device=flat.device)
        dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
        return out
    parts = [torch.empty(shape, dtype=flat.dtype, device=flat.device) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    return torch.cat(parts)


def gather_outputs(local, batch: int, queries: int, heads: int, group=None):
    """All-gather the local shards into full ``[B,SQ,H,512]`` / ``[B,1,SQ,H]``."""
    total = batch * queries
    world = dist.get_world_size(group)
    per = -(-total // world)
    out, mx, sm = (_all_gather(t, per, group)[:total] for t in local)
    return (out.reshape(batch, queries, heads, 512), mx.reshape(batch, 1, queries, heads),
            sm.reshape(batch, 1, queries, heads))


def sharded_forward(q, kv, q_rope, k_rope, indices, group=None, fn: Callable = None):
    """Each rank computes its query shard with ``fn`` (default
    ``dsa_b200.forward``) and all ranks receive the full outputs."""
    if fn is None:
        from .api import forward as fn
    batch, queries, heads, _ = q.shape
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = shard_bounds(batch * queries, world, rank)
    local = assemble_local(forward_pieces(q, kv, q_rope, k_rope, indices, lo, hi, fn), heads, q.device)
    return gather_outputs(local, batch, queries, heads, group)
