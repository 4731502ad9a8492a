"""Vendor-operator-shaped entry point for callers of the sparse flash
attention operator.

The reference benchmarks its kernel against the Ascend operator, called as
``npu_sparse_flash_attention(q, kv, kv, ids, 576 ** -0.5, query_rope=qr,
key_rope=kr, attention_mode=2, sparse_mode=0, return_softmax_lse=True)``
(tools/review.py:64-69). Its documented meaning (FAIRNESS_AUDIT.md:30-37):
``attention_mode=2`` is MLA absorb (the key tensor is also the value),
``sparse_mode=0`` adds no causal mask, ``return_softmax_lse=True`` asks for
the softmax max and sum (not a log-sum-exp tensor), BSND layouts.

``sparse_flash_attention`` accepts that call and runs the same sm_100a
forward as ``dsa_b200.forward``; the configuration the reference uses is the
one supported, and every other value of a mode, layout or optional input
raises ``ValueError`` instead of being ignored.
"""
from __future__ import annotations

import torch

from . import api

SUPPORTED_LAYOUT = "BSND"


def sparse_flash_attention(query, key, value, sparse_indices, scale_value, *,
                           block_table=None, actual_seq_lengths_query=None,
                           actual_seq_lengths_kv=None, query_rope=None, key_rope=None,
                           sparse_block_size=1, layout_query=SUPPORTED_LAYOUT,
                           layout_kv=SUPPORTED_LAYOUT, sparse_mode=0, attention_mode=2,
                           return_softmax_lse=False):
    """Sparse MLA attention in the vendor operator's argument order.

    query ``[B,SQ,H,512]``, key = value ``[B,L,1,512]``, sparse_indices
    ``[B,SQ,1,TOPK]`` int32, query_rope ``[B,SQ,H,64]``, key_rope
    ``[B,L,1,64]``; ``scale_value`` multiplies q.k + q_rope.k_rope and must
    lie in (0, 0.5]. Returns ``(attention_out, softmax_max, softmax_sum)``;
    with ``return_softmax_lse=False`` the two statistics are returned as
    empty FP32 tensors.
    """
    if attention_mode != 2:
        raise ValueError("only attention_mode=2 (MLA absorb: value is the key tensor) is supported")
    if sparse_mode != 0:
        raise ValueError("only sparse_mode=0 (no extra mask) is supported")
    if layout_query != SUPPORTED_LAYOUT or layout_kv != SUPPORTED_LAYOUT:
        raise ValueError(f"only {SUPPORTED_LAYOUT} layouts are supported")
    if sparse_block_size != 1:
        raise ValueError("only sparse_block_size=1 (one kv row per index) is supported")
    if block_table is not None:
        raise ValueError("a paged KV cache (block_table) is not supported")
    if actual_seq_lengths_query is not None or actual_seq_lengths_kv is not None:
        raise ValueError("ragged sequence lengths are not supported; mask with indices outside [0, L)")
    if query_rope is None or key_rope is None:
        raise ValueError("query_rope and key_rope are required (the scores span 512 + 64 dims)")
    if not isinstance(key, torch.Tensor) or not isinstance(value, torch.Tensor):
        raise ValueError("key and value must be tensors")
    same_view = (value.device == key.device and value.device.type != "meta"
                 and value.data_ptr() == key.data_ptr() and value.shape == key.shape
                 and value.stride() == key.stride() and value.dtype == key.dtype)
    if value is not key and not same_view:
        raise ValueError("attention_mode=2 reads the values from the key tensor: pass the same tensor")
    if isinstance(scale_value, bool) or not isinstance(scale_value, (int, float)):
        raise ValueError("scale_value must be a float")
    output, softmax_max, softmax_sum = api.forward(query, key, query_rope, key_rope, sparse_indices,
                                                   scale=float(scale_value))
    if not return_softmax_lse:
        empty = torch.empty((0,), dtype=torch.float32, device=output.device)
        return output, empty, empty.clone()
    return output, softmax_max, softmax_sum


# The vendor operator's name, for a one-line switch of the import.
npu_sparse_flash_attention = sparse_flash_attention
