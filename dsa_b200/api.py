"""Public entry point: check inputs, pick the launch entry, allocate, launch.

Mirrors ``forward`` of CHNJZ/dsa (dsa/api.py:76-132) on CUDA tensors:
same signature, same input contract (dsa/api.py:18-38), same outputs and the
same exception types. The device work is the sm_100a library
(libdsa_b200.so, include/dsa_b200.h) reached through ctypes; there is no
Python, Triton or CPU fallback.
"""
from __future__ import annotations

import ctypes
from collections import namedtuple

import torch

from . import _native
from .config import Tuning, select

# Device type the inputs must live on. Host-contract tests set it to "meta"
# (as tools/check_host_api.py:58 does for "npu") together with a stub
# launcher; product code never changes it.
DEVICE_TYPE = "cuda"

LaunchRecord = namedtuple("LaunchRecord", "name family heads_per_cta keys_per_tile split")

_FAMILY_NAMES = {_native.FAMILY_WARP_MMA: "warp_mma", _native.FAMILY_UMMA: "umma",
                 _native.FAMILY_UMMA_PAIR: "umma_pair", _native.FAMILY_STREAM: "stream",
                 _native.FAMILY_KEYS: "keys", _native.FAMILY_PAIR_UNION: "pair_union"}


def _check_inputs(q, kv, q_rope, k_rope, indices):
    """Shape/device/contiguity/dtype contract of dsa/api.py:18-38."""
    q_shape, kv_shape, ids_shape = q.shape, kv.shape, indices.shape
    if len(q_shape) != 4 or len(kv_shape) != 4 or len(ids_shape) != 4:
        raise ValueError("q, kv and indices must be 4-D tensors")
    batch, queries, heads, width = q_shape
    length, topk = kv_shape[1], ids_shape[-1]
    if (width != 512 or kv_shape != (batch, length, 1, 512) or q_rope.shape != (batch, queries, heads, 64)
            or k_rope.shape != (batch, length, 1, 64) or ids_shape != (batch, queries, 1, topk)
            or min(batch, queries, heads, length, topk) <= 0):
        raise ValueError("need q[B,SQ,H,512], kv[B,L,1,512], q_rope/k_rope with 64 dims, indices[B,SQ,1,K]")
    device = q.device
    if (device.type != DEVICE_TYPE or kv.device != device or q_rope.device != device
            or k_rope.device != device or indices.device != device or not q.is_contiguous()
            or not kv.is_contiguous() or not q_rope.is_contiguous() or not k_rope.is_contiguous()
            or not indices.is_contiguous()):
        raise ValueError("all inputs must be contiguous and on the same CUDA device")
    bf16 = torch.bfloat16
    if (q.dtype != bf16 or kv.dtype != bf16 or q_rope.dtype != bf16 or k_rope.dtype != bf16
            or indices.dtype != torch.int32):
        raise ValueError("q/kv/q_rope/k_rope must be bfloat16 and indices int32")
    return (batch, queries, heads, length, topk), device


def _check_cores(cores):
    # Accepted for source compatibility (dsa/api.py:76, :94-95); the grid is
    # sized from the device's SM count, so the value is only validated.
    if type(cores) is not int or cores <= 0:
        raise ValueError("cores must be a positive int")


SCALE_MAX = 0.5


def _check_scale(scale):
    """``None`` keeps the reference's fixed 1/sqrt(576) = 1/24 (0.0 at the C
    ABI); otherwise a real number in (0, 0.5] (every 1/sqrt(d) with d >= 4;
    larger scales would overflow the kernels' masked-key arithmetic)."""
    if scale is None:
        return 0.0
    if isinstance(scale, bool) or not isinstance(scale, (int, float)):
        raise ValueError("scale must be None or a float")
    value = float(scale)
    if not (0.0 < value <= SCALE_MAX):
        raise ValueError(f"scale must be in (0, {SCALE_MAX}], got {value}")
    return value


def _check_tuning(config, shape, cores):
    """Launch-entry checks: the reference's field rules (dsa/api.py:41-60)
    plus what the sm_100a kernels support (dsa_check_launch)."""
    if not isinstance(config, Tuning):
        raise TypeError("config must be a dsa_b200.Tuning")
    _, _, heads, _, _ = shape
    _check_cores(cores)
    if any(type(v) is not int or v <= 0 for v in (config.bm, config.bn, config.split, config.pv_cols)):
        raise ValueError("bm/bn/split/pv_cols must be positive ints")
    if config.bm not in (16, 32, 64, 128) or heads % config.bm:
        raise ValueError("bm must be 16/32/64/128 and divide the head count")
    if config.pv_cols not in (128, 256, 512):
        raise ValueError("pv_cols must be 128/256/512")


def _launch_from_tuning(config, shape):
    if config.bm == 128:
        family = _native.FAMILY_UMMA_PAIR if config.pv_cols == 512 else _native.FAMILY_UMMA
        launch = _native.Launch(family, 128, config.bn, config.split)
    elif config.bn == 32 and config.pv_cols == 128:
        launch = _native.Launch(_native.FAMILY_PAIR_UNION, 128, config.bn, config.split)
    elif config.bn == 32:
        launch = _native.Launch(_native.FAMILY_STREAM, 16, config.bn, config.split)
    elif config.pv_cols == 128:
        launch = _native.Launch(_native.FAMILY_KEYS, 16, config.bn, config.split)
    else:
        launch = _native.Launch(_native.FAMILY_WARP_MMA, 16, config.bn, config.split)
    code = _native.load().dsa_check_launch(*shape, ctypes.byref(launch))
    if code != _native.STATUS_OK:
        raise ValueError(f"Tuning {config} is not supported on sm_100a for shape {shape}: "
                         f"{_native.status_string(code)}")
    return launch


_default_cache = {}


def _default_launch(shape, device):
    key = (shape, device.index)
    launch = _default_cache.get(key)
    if launch is None:
        tuned = select(shape)
        if tuned is not None:
            launch = _launch_from_tuning(tuned, shape)
        else:
            launch = _native.Launch()
            code = _native.load().dsa_default_launch(*shape, ctypes.byref(launch))
            _native.raise_for_status(code, f"no launch entry for shape {shape}")
        _default_cache[key] = launch
    return launch


_status_words = {}


def _status_word(device):
    word = _status_words.get(device.index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=device)
        _status_words[device.index] = word
    return word


def _device_arg(device):
    return torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)


def device_status(device=None) -> int:
    """Synchronise and return the OR of device error bits reported so far
    (1 = a bounded device-side wait timed out)."""
    device = _device_arg(device)
    word = _status_word(device)
    torch.cuda.synchronize(device)
    return int(word.item())


def check_device_status(device=None) -> None:
    """Synchronise and raise ``RuntimeError`` (the C ABI's
    DSA_STATUS_DEVICE_TIMEOUT) if a kernel reported an error bit."""
    bits = device_status(device)
    if bits:
        raise RuntimeError(f"sparse-MLA kernel: {_native.status_string(_native.STATUS_DEVICE_TIMEOUT)} "
                           f"(device error bits {bits:#x})")


def clear_device_status(device=None) -> None:
    """Reset the device error word (kernels only ever set bits in it)."""
    device = _device_arg(device)
    _status_word(device).zero_()
    torch.cuda.synchronize(device)


def _launch_native(args, stream_handle):
    """Enqueue the forward through the C ABI; returns the kernel count."""
    lib = _native.load()
    code = lib.dsa_sparse_mla_fwd(ctypes.byref(args), stream_handle)
    _native.raise_for_status(code, "dsa_sparse_mla_fwd")
    return lib.dsa_last_launch_count()


def _workspace_bytes(args):
    return int(_native.load().dsa_fwd_workspace_bytes(ctypes.byref(args)))


def forward(q, kv, q_rope, k_rope, indices, *, config=None, cores=28, return_kernels=False,
            scale=None):
    """Sparse MLA attention with given top-k indices.

    Returns ``(output, softmax_max, softmax_sum)``: output BF16
    ``[B,SQ,H,512]``; the two statistics FP32 ``[B,1,SQ,H]`` (natural-exp
    max and sum of the scaled scores). The scale is the reference's fixed
    1/sqrt(512+64) unless ``scale`` gives one in (0, 0.5] (the reference
    fixes 1/24 and notes that a model keeps its own scale, README.md:81-84).
    Duplicate indices keep their repeated weight; indices outside [0, L) are
    masked. The reference requires at least one valid index per query
    (dsa/api.py:77-86); here a (query, head) row without one gets output 0,
    softmax_max -inf and softmax_sum 0.

    ``config`` overrides the shape-keyed launch entry; ``cores`` is validated
    for compatibility; ``return_kernels=True`` returns
    ``(outputs, launch_records)`` describing the enqueued kernels.
    Work is enqueued on ``torch.cuda.current_stream()``; nothing synchronises.
    """
    shape, device = _check_inputs(q, kv, q_rope, k_rope, indices)
    scale_arg = _check_scale(scale)
    if config is None:
        _check_cores(cores)
        launch = _default_launch(shape, device)
    else:
        _check_tuning(config, shape, cores)
        launch = _launch_from_tuning(config, shape)
    batch, queries, heads, length, topk = shape

    output = torch.empty_like(q)
    maximum = torch.empty((batch, 1, queries, heads), device=device, dtype=torch.float32)
    denominator = torch.empty_like(maximum)

    args = _native.FwdArgs()
    args.q, args.kv, args.q_rope, args.k_rope = q.data_ptr(), kv.data_ptr(), q_rope.data_ptr(), k_rope.data_ptr()
    args.indices = indices.data_ptr()
    args.output, args.softmax_max, args.softmax_sum = output.data_ptr(), maximum.data_ptr(), denominator.data_ptr()
    args.batch, args.queries, args.heads, args.length, args.topk = shape
    args.launch = launch
    args.scale = scale_arg
    ws_bytes = _workspace_bytes(args)
    workspace = None
    if ws_bytes:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        args.workspace, args.workspace_bytes = workspace.data_ptr(), ws_bytes
    args.status = _status_word(device).data_ptr()
    stream = torch.cuda.current_stream(device).cuda_stream if DEVICE_TYPE == "cuda" else 0
    count = _launch_native(args, stream)
    result = (output, maximum, denominator)
    if return_kernels:
        return result, _launch_records(launch, count)
    return result


def _launch_records(launch, count):
    """Descriptors of the kernels one call enqueued, in launch order: the
    union build before the union launch's pair kernel; the split merge after
    a main kernel with split > 1, unless the main kernel merged its partials
    itself (the split-V and stream families' cluster merge: one kernel)."""
    name = "dsa_fwd_" + _FAMILY_NAMES.get(launch.family, str(launch.family))
    fields = (launch.family, launch.heads_per_cta, launch.keys_per_tile, launch.split)
    if launch.family == _native.FAMILY_PAIR_UNION:
        names = ["dsa_union_build", name]
    elif launch.split > 1 and not (launch.family in (_native.FAMILY_UMMA, _native.FAMILY_STREAM) and count == 1):
        names = [name, "dsa_merge"]
    else:
        names = [name]
    if len(names) != count:
        raise RuntimeError(f"library enqueued {count} kernels, expected {names}")
    return tuple(LaunchRecord(n, *fields) for n in names)


def _check_paged(q, kv_cache, q_rope, k_rope_cache, block_table, indices, seq_lens):
    """Contract of forward_paged: q/q_rope/indices as for forward; the caches
    are page pools [NB, BS, 1, 512] / [NB, BS, 1, 64] BF16; block_table
    [B, MB] int32; seq_lens [B] int32 or None; all contiguous on one CUDA
    device."""
    if len(q.shape) != 4 or len(indices.shape) != 4 or len(kv_cache.shape) != 4 or len(block_table.shape) != 2:
        raise ValueError("q, kv_cache and indices must be 4-D tensors and block_table 2-D")
    batch, queries, heads, width = q.shape
    num_blocks, block_size = kv_cache.shape[0], kv_cache.shape[1]
    topk = indices.shape[-1]
    if (width != 512 or q_rope.shape != (batch, queries, heads, 64) or indices.shape != (batch, queries, 1, topk)
            or kv_cache.shape != (num_blocks, block_size, 1, 512)
            or k_rope_cache.shape != (num_blocks, block_size, 1, 64) or block_table.shape[0] != batch
            or min(batch, queries, heads, topk, num_blocks, block_size, block_table.shape[1]) <= 0
            or (seq_lens is not None and tuple(seq_lens.shape) != (batch,))):
        raise ValueError("need q[B,SQ,H,512], q_rope[B,SQ,H,64], indices[B,SQ,1,K], kv_cache[NB,BS,1,512], "
                         "k_rope_cache[NB,BS,1,64], block_table[B,MB], seq_lens[B]")
    device = q.device
    tensors = [q, kv_cache, q_rope, k_rope_cache, block_table, indices] + ([seq_lens] if seq_lens is not None else [])
    if device.type != DEVICE_TYPE or any(t.device != device or not t.is_contiguous() for t in tensors):
        raise ValueError("all inputs must be contiguous and on the same CUDA device")
    bf16 = torch.bfloat16
    if (q.dtype != bf16 or kv_cache.dtype != bf16 or q_rope.dtype != bf16 or k_rope_cache.dtype != bf16
            or indices.dtype != torch.int32 or block_table.dtype != torch.int32
            or (seq_lens is not None and seq_lens.dtype != torch.int32)):
        raise ValueError("q/kv_cache/q_rope/k_rope_cache must be bfloat16; indices, block_table, seq_lens int32")
    if num_blocks * block_size > 0x7fffffff:
        raise ValueError("the page pool holds more than 2^31 - 1 rows")
    return (batch, queries, heads, topk, num_blocks, block_size, block_table.shape[1]), device


def forward_paged(q, kv_cache, q_rope, k_rope_cache, block_table, indices, *, seq_lens=None, config=None,
                  cores=28, scale=None):
    """``forward`` over a paged KV cache.

    ``kv_cache`` / ``k_rope_cache`` are page pools ``[NB, BS, 1, 512]`` /
    ``[NB, BS, 1, 64]``; ``block_table[b, j]`` is the pool block holding
    tokens ``[j*BS, (j+1)*BS)`` of batch row ``b``; ``indices`` are logical
    token positions. An index is masked when negative, at or past
    ``seq_lens[b]`` (or ``MB * BS``), or when its table entry is outside
    ``[0, NB)``. The result equals ``forward`` on the dense cache that the
    table describes (same kernels, same arithmetic). The reference has no
    paged layout (README.md:19-20); this is the adjacent KV-cache format.
    """
    (batch, queries, heads, topk, num_blocks, block_size, max_blocks), device = _check_paged(
        q, kv_cache, q_rope, k_rope_cache, block_table, indices, seq_lens)
    scale_arg = _check_scale(scale)
    inner = (1, batch * queries, heads, num_blocks * block_size, topk)
    if config is None:
        _check_cores(cores)
        launch = _default_launch(inner, device)
    else:
        _check_tuning(config, inner, cores)
        launch = _launch_from_tuning(config, inner)
    output = torch.empty_like(q)
    maximum = torch.empty((batch, 1, queries, heads), device=device, dtype=torch.float32)
    denominator = torch.empty_like(maximum)
    args = _native.FwdArgs()
    args.q, args.kv, args.q_rope, args.k_rope = q.data_ptr(), kv_cache.data_ptr(), q_rope.data_ptr(), k_rope_cache.data_ptr()
    args.indices = indices.data_ptr()
    args.output, args.softmax_max, args.softmax_sum = output.data_ptr(), maximum.data_ptr(), denominator.data_ptr()
    args.batch, args.queries, args.heads, args.length, args.topk = batch, queries, heads, num_blocks * block_size, topk
    args.launch = launch
    args.scale = scale_arg
    paged = _native.PagedKv(block_table.data_ptr(), seq_lens.data_ptr() if seq_lens is not None else None,
                            max_blocks, block_size, num_blocks)
    lib = _native.load()
    ws_bytes = int(lib.dsa_fwd_paged_workspace_bytes(ctypes.byref(args), ctypes.byref(paged)))
    if ws_bytes == 0:
        raise ValueError(f"no launch entry for the paged shape {inner}")
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    args.workspace, args.workspace_bytes = workspace.data_ptr(), ws_bytes
    args.status = _status_word(device).data_ptr()
    stream = torch.cuda.current_stream(device).cuda_stream if DEVICE_TYPE == "cuda" else 0
    code = lib.dsa_sparse_mla_fwd_paged(ctypes.byref(args), ctypes.byref(paged), stream)
    _native.raise_for_status(code, "dsa_sparse_mla_fwd_paged")
    return output, maximum, denominator


FP8_WORKSPACE_BUDGET = 1 << 30  # bytes of dequantised rows per dsa_sparse_mla_fwd_fp8 call


def forward_fp8(q, kv_fp8, q_rope, indices, *, config=None, cores=28, scale=None):
    """``forward`` over an FP8 KV cache (DeepSeek-V3.2's FP8 MLA layout).

    ``kv_fp8`` is uint8 ``[B, L, 1, 656]`` per token: 512 float8 e4m3
    latent values, 4 FP32 scales (one per 128 latent dims), 64 BF16 rope
    dims (see ``quantize_kv_fp8``). Each query's selected rows are
    dequantised (``bf16(e4m3 * scale)``) into a workspace by one kernel and
    the BF16 forward runs on them, in pieces of whole queries that keep the
    workspace under ``FP8_WORKSPACE_BUDGET``. The reference keeps kv in BF16
    and leaves quantised caches out (DSA从原理到实现.md:626).
    """
    if len(q.shape) != 4 or len(kv_fp8.shape) != 4 or len(indices.shape) != 4:
        raise ValueError("q, kv_fp8 and indices must be 4-D tensors")
    batch, queries, heads, width = q.shape
    length, topk = kv_fp8.shape[1], indices.shape[-1]
    if (width != 512 or kv_fp8.shape != (batch, length, 1, _native.FP8_ROW_BYTES)
            or q_rope.shape != (batch, queries, heads, 64) or indices.shape != (batch, queries, 1, topk)
            or min(batch, queries, heads, length, topk) <= 0):
        raise ValueError("need q[B,SQ,H,512], kv_fp8[B,L,1,656] uint8, q_rope[B,SQ,H,64], indices[B,SQ,1,K]")
    device = q.device
    if (device.type != DEVICE_TYPE or any(t.device != device or not t.is_contiguous()
                                          for t in (q, kv_fp8, q_rope, indices))):
        raise ValueError("all inputs must be contiguous and on the same CUDA device")
    if (q.dtype != torch.bfloat16 or q_rope.dtype != torch.bfloat16 or kv_fp8.dtype != torch.uint8
            or indices.dtype != torch.int32):
        raise ValueError("q/q_rope must be bfloat16, kv_fp8 uint8 and indices int32")
    scale_arg = _check_scale(scale)
    if config is not None:
        _check_tuning(config, (batch * queries, 1, heads, topk, topk), cores)
    else:
        _check_cores(cores)
    output = torch.empty_like(q)
    maximum = torch.empty((batch, 1, queries, heads), device=device, dtype=torch.float32)
    denominator = torch.empty_like(maximum)
    lib = _native.load()
    stream = torch.cuda.current_stream(device).cuda_stream if DEVICE_TYPE == "cuda" else 0
    per_query = topk * (1024 + 128 + 4)
    chunk = max(1, min(queries, FP8_WORKSPACE_BUDGET // per_query))
    rows_per_batch = length * _native.FP8_ROW_BYTES
    for b in range(batch):
        for s0 in range(0, queries, chunk):
            n = min(chunk, queries - s0)
            t0 = b * queries + s0
            shape = (n, 1, heads, topk, topk)  # the inner forward's shape
            launch = _launch_from_tuning(config, shape) if config is not None else _default_launch(shape, device)
            args = _native.FwdArgs()
            args.q = q.data_ptr() + t0 * heads * 512 * 2
            args.q_rope = q_rope.data_ptr() + t0 * heads * 64 * 2
            args.kv = kv_fp8.data_ptr() + b * rows_per_batch
            args.k_rope = None
            args.indices = indices.data_ptr() + t0 * topk * 4
            args.output = output.data_ptr() + t0 * heads * 512 * 2
            args.softmax_max = maximum.data_ptr() + t0 * heads * 4
            args.softmax_sum = denominator.data_ptr() + t0 * heads * 4
            args.batch, args.queries, args.heads, args.length, args.topk = 1, n, heads, length, topk
            args.launch = launch
            args.scale = scale_arg
            ws_bytes = int(lib.dsa_fwd_fp8_workspace_bytes(ctypes.byref(args)))
            if ws_bytes == 0:
                raise ValueError(f"no launch entry for the FP8 shape {shape}")
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
            args.workspace, args.workspace_bytes = workspace.data_ptr(), ws_bytes
            args.status = _status_word(device).data_ptr()
            code = lib.dsa_sparse_mla_fwd_fp8(ctypes.byref(args), stream)
            _native.raise_for_status(code, "dsa_sparse_mla_fwd_fp8")
    return output, maximum, denominator


class ForwardPlan:
    """``forward`` prepared once for fixed input tensors.

    Checks the inputs, picks the launch entry and allocates the outputs and
    the split-KV workspace at construction; ``run()`` then only enqueues the
    kernels on the current stream (no allocation, no host synchronisation),
    so a serving loop can call it per step or capture it in a CUDA graph.
    The plan keeps references to its inputs: callers update them in place
    (same addresses) between runs. Results are written into the same
    ``(output, softmax_max, softmax_sum)`` tensors every run.
    """

    def __init__(self, q, kv, q_rope, k_rope, indices, *, config=None, cores=28, scale=None):
        shape, device = _check_inputs(q, kv, q_rope, k_rope, indices)
        scale_arg = _check_scale(scale)
        if config is None:
            _check_cores(cores)
            launch = _default_launch(shape, device)
        else:
            _check_tuning(config, shape, cores)
            launch = _launch_from_tuning(config, shape)
        batch, queries, heads, _, _ = shape
        self.inputs = (q, kv, q_rope, k_rope, indices)
        self.device = device
        self.launch = launch
        self.outputs = (torch.empty_like(q),
                        torch.empty((batch, 1, queries, heads), device=device, dtype=torch.float32),
                        torch.empty((batch, 1, queries, heads), device=device, dtype=torch.float32))
        args = _native.FwdArgs()
        args.q, args.kv, args.q_rope, args.k_rope = q.data_ptr(), kv.data_ptr(), q_rope.data_ptr(), k_rope.data_ptr()
        args.indices = indices.data_ptr()
        args.output, args.softmax_max, args.softmax_sum = (t.data_ptr() for t in self.outputs)
        args.batch, args.queries, args.heads, args.length, args.topk = shape
        args.launch = launch
        args.scale = scale_arg
        ws_bytes = _workspace_bytes(args)
        self.workspace = None
        if ws_bytes:
            self.workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
            args.workspace, args.workspace_bytes = self.workspace.data_ptr(), ws_bytes
        args.status = _status_word(device).data_ptr()
        self._args = args
        self._args_ref = ctypes.byref(args)
        self._lib = _native.load()
        self.kernels = None  # kernels per run, known after the first run

    def run(self):
        """Enqueue one forward on the current stream; returns the output tensors."""
        stream = torch.cuda.current_stream(self.device).cuda_stream if DEVICE_TYPE == "cuda" else 0
        code = self._lib.dsa_sparse_mla_fwd(self._args_ref, stream)
        if code != _native.STATUS_OK:
            _native.raise_for_status(code, "dsa_sparse_mla_fwd")
        self.kernels = self._lib.dsa_last_launch_count()
        return self.outputs
