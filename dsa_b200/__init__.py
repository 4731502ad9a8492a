"""B200 (sm_100a) sparse-MLA attention forward with the CHNJZ/dsa API.

Drop-in for ``dsa.forward`` (dsa/__init__.py:2-5 of the reference):
``import dsa_b200 as dsa; dsa.forward(q, kv, q_rope, k_rope, indices)``.
"""
from .api import (ForwardPlan, check_device_status, clear_device_status, device_status, forward, forward_fp8,
                  forward_paged)
from .fp8_cache import quantize_kv_fp8
from .indexer import indexer_topk
from .config import CASE_SHAPES, SELECTED, Tuning
from .sparse_flash_attention import npu_sparse_flash_attention, sparse_flash_attention

__all__ = ["forward", "forward_paged", "forward_fp8", "quantize_kv_fp8", "indexer_topk", "ForwardPlan", "Tuning", "CASE_SHAPES", "SELECTED", "device_status",
           "check_device_status", "clear_device_status", "sparse_flash_attention",
           "npu_sparse_flash_attention"]
