"""Lightning indexer + top-k: the indices of the sparse-MLA forward.

``indexer_topk(q_idx, k_idx, weights, topk)`` computes, for every query t
of batch row b and key j < L,
``score[t, j] = sum_h weights[t, h] * relu(q_idx[t, h] . k_idx[b, j])`` on
the tensor cores (BF16 products, FP32 sums) and returns the ``topk`` keys
with the largest scores as int32 ``[B, SQ, 1, topk]`` in ascending key order
(ties to the smaller key; padded with -1 when a query has fewer than
``topk`` valid keys), the index layout ``forward`` takes. ``lengths``
(int32 ``[B, SQ]``) limits each query to keys ``j < lengths[b, s]`` (a
causal prefill passes position + 1). The reference takes the indices as
given and leaves this stage out (README.md:19-20); this is DeepSeek-V3.2's
indexer formula.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native
from .api import DEVICE_TYPE, _status_word

INDEX_DIM = 128
SCORE_BUDGET = 1 << 30  # bytes of FP32 scores per library call when they are not returned


def indexer_topk(q_idx, k_idx, weights, topk, *, lengths=None, return_scores=False):
    if len(q_idx.shape) != 4 or len(k_idx.shape) != 3 or len(weights.shape) != 3:
        raise ValueError("need q_idx[B,SQ,HI,128], k_idx[B,L,128], weights[B,SQ,HI]")
    batch, queries, heads, dim = q_idx.shape
    length = k_idx.shape[1]
    if (dim != INDEX_DIM or k_idx.shape != (batch, length, INDEX_DIM) or weights.shape != (batch, queries, heads)
            or heads not in (16, 32, 64, 128) or type(topk) is not int or topk <= 0
            or (lengths is not None and tuple(lengths.shape) != (batch, queries))):
        raise ValueError("need q_idx[B,SQ,HI,128] (HI 16/32/64/128), k_idx[B,L,128], weights[B,SQ,HI], "
                         "lengths[B,SQ], topk > 0")
    device = q_idx.device
    tensors = [q_idx, k_idx, weights] + ([lengths] if lengths is not None else [])
    if device.type != DEVICE_TYPE or any(t.device != device or not t.is_contiguous() for t in tensors):
        raise ValueError("all inputs must be contiguous and on the same CUDA device")
    if (q_idx.dtype != torch.bfloat16 or k_idx.dtype != torch.bfloat16 or weights.dtype != torch.float32
            or (lengths is not None and lengths.dtype != torch.int32)):
        raise ValueError("q_idx/k_idx must be bfloat16, weights float32, lengths int32")
    indices = torch.empty((batch, queries, 1, topk), dtype=torch.int32, device=device)
    scores = torch.empty((batch, queries, length), dtype=torch.float32, device=device) if return_scores else None
    lib = _native.load()
    stream = torch.cuda.current_stream(device).cuda_stream if DEVICE_TYPE == "cuda" else 0
    # one call when the scores fit SCORE_BUDGET (or are returned); otherwise
    # pieces of whole batch rows, or of whole queries of one batch row
    if return_scores or batch * queries * length * 4 <= SCORE_BUDGET:
        pieces = [(0, batch, 0, queries)]
    elif queries * length * 4 <= SCORE_BUDGET:
        rows = max(1, SCORE_BUDGET // (queries * length * 4))
        pieces = [(b0, min(batch, b0 + rows), 0, queries) for b0 in range(0, batch, rows)]
    else:
        chunk = max(1, SCORE_BUDGET // (length * 4))
        pieces = [(b, b + 1, s0, min(queries, s0 + chunk)) for b in range(batch) for s0 in range(0, queries, chunk)]
    for b0, b1, s0, s1 in pieces:
        t0 = b0 * queries + s0
        a = _native.IndexerArgs()
        a.q = q_idx.data_ptr() + t0 * heads * INDEX_DIM * 2
        a.k = k_idx.data_ptr() + b0 * length * INDEX_DIM * 2
        a.weights = weights.data_ptr() + t0 * heads * 4
        a.lengths = lengths.data_ptr() + t0 * 4 if lengths is not None else None
        a.indices = indices.data_ptr() + t0 * topk * 4
        a.scores = scores.data_ptr() + t0 * length * 4 if return_scores else None
        a.batch, a.queries, a.heads, a.length, a.topk = b1 - b0, s1 - s0, heads, length, topk
        ws = int(lib.dsa_indexer_workspace_bytes(ctypes.byref(a)))
        buf = torch.empty(ws, dtype=torch.uint8, device=device) if ws else None
        a.workspace, a.workspace_bytes = (buf.data_ptr(), ws) if ws else (None, 0)
        a.status = _status_word(device).data_ptr()
        code = lib.dsa_indexer_topk(ctypes.byref(a), stream)
        _native.raise_for_status(code, "dsa_indexer_topk")
    return (indices, scores) if return_scores else indices
