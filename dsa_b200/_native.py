"""ctypes binding of libdsa_b200.so (the C ABI in include/dsa_b200.h).

The library is loaded lazily on first use and never replaced by a Python or
CPU fallback: if it is missing or was built for another ABI version, every
call raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading

ABI_VERSION = 2
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdsa_b200.so")

STATUS_OK = 0
STATUS_BAD_ARGUMENT = 1
STATUS_UNSUPPORTED = 2
STATUS_WORKSPACE_TOO_SMALL = 3
STATUS_LAUNCH_FAILED = 4
STATUS_DEVICE_TIMEOUT = 5
STATUS_CUDA_ERROR = 6

FAMILY_AUTO = 0
FAMILY_WARP_MMA = 1
FAMILY_UMMA = 2
FAMILY_UMMA_PAIR = 3
FAMILY_STREAM = 4
FAMILY_KEYS = 5
FAMILY_PAIR_UNION = 6

# Every entry point declared in include/dsa_b200.h.
EXPORTS = (
    "dsa_abi_version",
    "dsa_status_string",
    "dsa_default_launch",
    "dsa_check_launch",
    "dsa_fwd_workspace_bytes",
    "dsa_sparse_mla_fwd",
    "dsa_merge_partials",
    "dsa_last_launch_count",
    "dsa_sparse_mla_fwd_noalloc",
    "dsa_set_wait_test",
    "dsa_fwd_paged_workspace_bytes",
    "dsa_sparse_mla_fwd_paged",
    "dsa_fwd_fp8_workspace_bytes",
    "dsa_sparse_mla_fwd_fp8",
    "dsa_indexer_workspace_bytes",
    "dsa_indexer_topk",
)

# Bytes per token of the FP8 KV cache (DSA_FP8_ROW_BYTES in include/dsa_b200.h).
FP8_ROW_BYTES = 656

# Byte size of the built-in scratch array of dsa_sparse_mla_fwd_noalloc
# (DSA_NOALLOC_SCRATCH_BYTES in include/dsa_b200.h).
NOALLOC_SCRATCH_BYTES = 32 << 20


class Launch(ctypes.Structure):
    _fields_ = [("family", ctypes.c_int32), ("heads_per_cta", ctypes.c_int32),
                ("keys_per_tile", ctypes.c_int32), ("split", ctypes.c_int32)]


class PagedKv(ctypes.Structure):
    _fields_ = [("block_table", ctypes.c_void_p), ("seq_lens", ctypes.c_void_p),
                ("max_blocks", ctypes.c_int64), ("block_size", ctypes.c_int64), ("num_blocks", ctypes.c_int64)]


class IndexerArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("weights", ctypes.c_void_p), ("lengths", ctypes.c_void_p),
        ("indices", ctypes.c_void_p), ("scores", ctypes.c_void_p),
        ("batch", ctypes.c_int64), ("queries", ctypes.c_int64), ("heads", ctypes.c_int64),
        ("length", ctypes.c_int64), ("topk", ctypes.c_int64),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64), ("status", ctypes.c_void_p),
    ]


class FwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("kv", ctypes.c_void_p), ("q_rope", ctypes.c_void_p),
        ("k_rope", ctypes.c_void_p), ("indices", ctypes.c_void_p), ("output", ctypes.c_void_p),
        ("softmax_max", ctypes.c_void_p), ("softmax_sum", ctypes.c_void_p),
        ("batch", ctypes.c_int64), ("queries", ctypes.c_int64), ("heads", ctypes.c_int64),
        ("length", ctypes.c_int64), ("topk", ctypes.c_int64),
        ("launch", Launch),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_uint64),
        ("status", ctypes.c_void_p),
        ("scale", ctypes.c_float),
    ]


_lib = None
_lock = threading.Lock()


def load():
    """Load the library once; raise RuntimeError if it is absent or stale."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the sm_100a library first "
                "(python -m dsa_b200.build or __graft_entry__.build()); there is no fallback")
        lib = _bind(ctypes.CDLL(LIB_PATH))
        version = lib.dsa_abi_version()
        if version != ABI_VERSION:
            raise RuntimeError(f"libdsa_b200.so ABI {version} != expected {ABI_VERSION}; rebuild it")
        _lib = lib
        return lib


CHECKED_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdsa_b200_checked.so")


def load_checked():
    """The bounds-checking debug build (same ABI; a failed check sets bit 4 of
    the status word). Raises RuntimeError when it has not been built."""
    if not os.path.exists(CHECKED_LIB_PATH):
        raise RuntimeError(f"{CHECKED_LIB_PATH} is missing: python -m dsa_b200.build --bounds-check")
    return _bind(ctypes.CDLL(CHECKED_LIB_PATH))


def _bind(lib):
    """Declare the prototypes of include/dsa_b200.h on a loaded library."""
    lib.dsa_abi_version.restype = ctypes.c_int
    lib.dsa_status_string.restype = ctypes.c_char_p
    lib.dsa_status_string.argtypes = [ctypes.c_int]
    lib.dsa_default_launch.restype = ctypes.c_int
    lib.dsa_default_launch.argtypes = [ctypes.c_int64] * 5 + [ctypes.POINTER(Launch)]
    lib.dsa_check_launch.restype = ctypes.c_int
    lib.dsa_check_launch.argtypes = [ctypes.c_int64] * 5 + [ctypes.POINTER(Launch)]
    lib.dsa_fwd_workspace_bytes.restype = ctypes.c_uint64
    lib.dsa_fwd_workspace_bytes.argtypes = [ctypes.POINTER(FwdArgs)]
    lib.dsa_sparse_mla_fwd.restype = ctypes.c_int
    lib.dsa_sparse_mla_fwd.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_void_p]
    lib.dsa_merge_partials.restype = ctypes.c_int
    lib.dsa_merge_partials.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]
    lib.dsa_last_launch_count.restype = ctypes.c_int
    lib.dsa_sparse_mla_fwd_noalloc.restype = ctypes.c_int
    lib.dsa_sparse_mla_fwd_noalloc.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_void_p]
    lib.dsa_fwd_paged_workspace_bytes.restype = ctypes.c_uint64
    lib.dsa_fwd_paged_workspace_bytes.argtypes = [ctypes.POINTER(FwdArgs), ctypes.POINTER(PagedKv)]
    lib.dsa_sparse_mla_fwd_paged.restype = ctypes.c_int
    lib.dsa_sparse_mla_fwd_paged.argtypes = [ctypes.POINTER(FwdArgs), ctypes.POINTER(PagedKv), ctypes.c_void_p]
    lib.dsa_fwd_fp8_workspace_bytes.restype = ctypes.c_uint64
    lib.dsa_fwd_fp8_workspace_bytes.argtypes = [ctypes.POINTER(FwdArgs)]
    lib.dsa_sparse_mla_fwd_fp8.restype = ctypes.c_int
    lib.dsa_sparse_mla_fwd_fp8.argtypes = [ctypes.POINTER(FwdArgs), ctypes.c_void_p]
    lib.dsa_indexer_workspace_bytes.restype = ctypes.c_uint64
    lib.dsa_indexer_workspace_bytes.argtypes = [ctypes.POINTER(IndexerArgs)]
    lib.dsa_indexer_topk.restype = ctypes.c_int
    lib.dsa_indexer_topk.argtypes = [ctypes.POINTER(IndexerArgs), ctypes.c_void_p]
    lib.dsa_set_wait_test.restype = ctypes.c_int
    lib.dsa_set_wait_test.argtypes = [ctypes.c_uint64, ctypes.c_int]
    return lib


def status_string(code: int) -> str:
    return load().dsa_status_string(int(code)).decode()


def raise_for_status(code: int, what: str) -> None:
    """Map a dsa_status_t to the reference's exception types (ValueError for
    argument/config problems, dsa/api.py:22-37; RuntimeError otherwise)."""
    if code == STATUS_OK:
        return
    msg = f"{what}: {status_string(code)} (status {code})"
    if code in (STATUS_BAD_ARGUMENT, STATUS_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)
