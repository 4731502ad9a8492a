#!/usr/bin/env python
"""Sparse-MLA forward benchmark on B200 (one process per GPU).

``python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME]
[--variant uniform|peaked|duplicates] [--impl ours|reference]
[--inputs device|reference]``

A step is one full ``dsa_b200.forward`` call (main kernel + merge when
split > 1) over the config's synthetic inputs. With N ranks (torchrun), the
flattened B*SQ queries are sharded contiguously (kv replicated per rank);
each rank times only its own forward calls; the reported time is the max
over ranks. The output all-gather runs after the timed region.

Default workload: ``prefill_h128`` (B=4, SQ=4096, H=128, L=65536,
TOPK=2048), the benchmark config that is partitioned across 1/2/4/8 B200.
Total work is fixed as N grows ("strong" scaling).

``--impl reference`` times the reference's own FP32 math (the CPU oracle,
tools/review.py:123-145 of CHNJZ/dsa) on all host cores, on a bounded
sample of the same workload per step, scaled to a full call.

Inputs are drawn on the device by default (same shapes and distributions as
the reference's generator, seconds even for prefill_h128); ``--inputs
reference`` draws them in the reference's own order on the CPU instead
(tools/review.py:35-61: one generator seeded with the config's seed, randn
for q, kv, q_rope, k_rope, then randperm(L)[:TOPK] per query), so the values
are the ones the reference's runs for that seed use (uniform variant only;
minutes of host time for prefill_h128).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "sparse-MLA fwd µs/call, HBM GB/s & TFLOP/s vs roofline at 1/2/4/8 B200"
SEED = 20261103

# name -> (B, SQ, H, L, TOPK); BASELINE.json configs[0..4]
CONFIGS = {
    "decode_b1": (1, 1, 128, 4096, 2048),
    "decode_b8": (8, 2, 128, 32768, 2048),
    "decode_tp8": (64, 1, 16, 65536, 2048),
    "prefill_tp8": (1, 4096, 16, 8192, 2048),
    "prefill_h128": (4, 4096, 128, 65536, 2048),
}
DEFAULT_CONFIG = "prefill_h128"

# Dominant-kernel DRAM traffic per launch (dram__bytes_read.sum +
# dram__bytes_write.sum), from one-pass ncu captures (`--cache-control none`)
# of timed-loop launches of this script, i.e. right after the 256 MiB write
# that flushes the L2: the writes include the flush buffer's dirty lines that
# the launch evicts (a decode launch writes back about as many bytes as it
# brings into the L2). Modelled per rank on the uniform index variant as
#   traffic = replicated + per_query * (queries of the rank)
# where `replicated` is what every rank reads whatever its query count (kv
# rows that stay L2-resident after their first read). The bench reports
# None for any other variant, shape or launch entry.
TRAFFIC_MODEL = {
    # fwd_pair_kernel, prefill_h128: 10.506 GB read + 2.239 GB written (the
    # 2.15 GB of outputs and the flush's dirty lines). kv is re-read in
    # proportion to the queries (75.5 MB of kv per batch row does not stay
    # in the L2 next to the streamed q and outputs), so it all scales per query.
    "prefill_h128": (0.0, (10.506e9 + 2.239e9) / 16384),
    # union launch's fwd_pair_kernel, prefill_tp8: 95.1 MB read + 84.1 MB
    # written (67 MB of outputs and dirty lines written back), of which the
    # 9.4 MB kv + k_rope is read once (it stays L2-resident) and the rest
    # scales with the queries.
    "prefill_tp8": (9.4e6, (95.1e6 + 84.1e6 - 9.4e6) / 4096),
    # fwd_stream_kernel (cluster merge), decode_tp8: 152.7 MB read + 61.6 MB
    # of dirty lines written back.
    "decode_tp8": (0.0, (152.7e6 + 61.6e6) / 64),
    # fwd_umma_kernel (cluster merge), decode_b8: 39.1 MB read + 33.2 MB
    # written back (the FP32 partials themselves stay in the L2).
    "decode_b8": (0.0, (39.1e6 + 33.2e6) / 16),
    # fwd_umma_kernel (cluster merge, split 16), decode_b1: 2.57 MB read +
    # 5.72 MB written back.
    "decode_b1": (0.0, 2.57e6 + 5.72e6),
}


def traffic_bytes(config, variant, custom, rank_queries):
    """Modelled DRAM bytes of one launch of the dominant kernel on a rank
    (None when no capture covers the workload)."""
    if custom or variant != "uniform" or config not in TRAFFIC_MODEL:
        return None
    replicated, per_query = TRAFFIC_MODEL[config]
    return int(replicated + per_query * rank_queries)


# The CPU oracle (the reference's FP32 math) is timed on the same bounded
# sample in both arms: the first CPU_SAMPLE_QUERIES flattened queries (all of
# them when the config has fewer), in chunks of 16 queries for H >= 64 and
# 128 otherwise, scaled to a full call.
CPU_SAMPLE_QUERIES = 1024

L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def algorithmic(shape):
    """Per-call algorithmic work: gathered bytes Q*TOPK*1152, other bytes
    (q, q_rope, output, stats, indices) and FLOPs Q*H*2*TOPK*1088."""
    b, s, h, _, k = shape
    q = b * s
    gathered = q * k * 1152
    other = q * h * (512 + 64) * 2 + q * h * 512 * 2 + q * h * 8 + q * k * 4
    flops = q * h * 2 * k * 1088
    return gathered, other, flops


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# Synthetic inputs (seeded, generated on the device; same shapes and value
# distributions as the configs: N(0,1) BF16 tensors, int32 indices).
# ---------------------------------------------------------------------------
def make_device_indices(batch, queries, length, topk, seed, variant, device):
    g = torch.Generator(device=device).manual_seed(seed + 1)
    rows = batch * queries
    out = torch.empty((rows, topk), dtype=torch.int32, device=device)
    if variant in ("uniform", "duplicates"):
        chunk = max(1, (256 << 20) // (length * 4))
        for r0 in range(0, rows, chunk):
            r1 = min(rows, r0 + chunk)
            keys = torch.rand((r1 - r0, length), generator=g, device=device)
            out[r0:r1] = keys.argsort(dim=-1)[:, :topk].int()
        if variant == "duplicates":
            n_dup = int(round(0.1 * topk))
            gc = torch.Generator().manual_seed(seed + 2)
            host = out.cpu()
            for r in range(rows):
                slots = (torch.randperm(topk - 1, generator=gc)[:n_dup] + 1).sort().values.tolist()
                row = host[r]
                for slot in slots:
                    row[slot] = row[int(torch.randint(0, slot, (1,), generator=gc))]
            out.copy_(host)
    elif variant == "peaked":
        recent = min(4096, length)
        n_hot = min(int(round(0.7 * topk)), recent)
        n_cold = topk - n_hot
        hot = torch.rand((rows, recent), generator=g, device=device).argsort(-1)[:, :n_hot] + (length - recent)
        cold = torch.rand((rows, length - recent), generator=g, device=device).argsort(-1)[:, :n_cold]
        out.copy_(torch.cat([hot, cold], dim=1).int())
    else:
        raise ValueError(variant)
    return out.reshape(batch, queries, 1, topk)


def make_reference_order_inputs(shape, seed=SEED, device="cuda"):
    """The inputs the reference's generator gives for ``seed``
    (tools/review.py:35-61): one CPU generator, N(0,1) draws for q, kv,
    q_rope and k_rope in that order (rounded to BF16), then
    randperm(L)[:TOPK] for every (b, s) in order; copied to ``device``."""
    b, s, h, length, k = shape
    g = torch.Generator().manual_seed(seed)

    def normal(*dims):
        return torch.randn(dims, generator=g).bfloat16().to(device)

    q = normal(b, s, h, 512)
    kv = normal(b, length, 1, 512)
    q_rope = normal(b, s, h, 64)
    k_rope = normal(b, length, 1, 64)
    ids = torch.empty((b * s, k), dtype=torch.int32)
    for r in range(b * s):
        ids[r] = torch.randperm(length, generator=g)[:k]
    return q, kv, q_rope, k_rope, ids.reshape(b, s, 1, k).to(device)


def make_inputs_for(args, shape, device):
    if args.inputs == "reference":
        if args.variant != "uniform":
            raise SystemExit("--inputs reference draws the reference's uniform indices only")
        return make_reference_order_inputs(shape, SEED, device)
    return make_device_inputs(shape, SEED, args.variant, device)


def make_device_inputs(shape, seed=SEED, variant="uniform", device="cuda"):
    b, s, h, length, k = shape
    g = torch.Generator(device=device).manual_seed(seed)

    def normal(*dims):
        t = torch.empty(dims, dtype=torch.bfloat16, device=device)
        flat = t.view(-1)
        step = 1 << 28
        for i in range(0, flat.numel(), step):
            n = min(step, flat.numel() - i)
            flat[i:i + n] = torch.randn(n, generator=g, device=device).bfloat16()
        return t

    q = normal(b, s, h, 512)
    kv = normal(b, length, 1, 512)
    q_rope = normal(b, s, h, 64)
    k_rope = normal(b, length, 1, 64)
    ids = make_device_indices(b, s, length, k, seed, variant, device)
    return q, kv, q_rope, k_rope, ids


def compact_for_oracle(data, rows):
    """CPU copies of the inputs restricted to flattened query ``rows``, with
    each query's selected kv rows gathered into its own compact batch
    (L' = TOPK, indices remapped, invalid ones kept invalid). The oracle's
    arithmetic on the compact problem is identical to the full one."""
    q, kv, q_rope, k_rope, ids = data
    b, s, h, _ = q.shape
    length = kv.shape[1]
    rows_t = torch.as_tensor(rows, device=q.device, dtype=torch.long)
    bi = rows_t // s
    si = rows_t % s
    idx = ids[bi, si, 0].long()                       # [n, K]
    valid = (idx >= 0) & (idx < length)
    safe = idx.clamp(0, length - 1)
    kv_c = kv[bi[:, None], safe, 0]                  # [n, K, 512]
    kr_c = k_rope[bi[:, None], safe, 0]
    k = idx.shape[1]
    ids_c = torch.arange(k, device=q.device, dtype=torch.int32).expand(len(rows), k).clone()
    ids_c[~valid] = -1
    return (q[bi, si].unsqueeze(1).cpu(), kv_c.unsqueeze(2).cpu(), q_rope[bi, si].unsqueeze(1).cpu(),
            kr_c.unsqueeze(2).cpu(), ids_c.reshape(len(rows), 1, 1, k).cpu())


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        # Address the GPU by UUID so the sample follows the CUDA device even
        # when CUDA_VISIBLE_DEVICES renumbers devices.
        try:
            uuid = str(torch.cuda.get_device_properties(gpu_index).uuid)
            self.gpu_index = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:  # noqa: BLE001 - fall back to the ordinal
            self.gpu_index = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, start, end):
        """Host wall-clock bounds of the timed region."""
        self.window = (start, end)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread is not None:
                self.thread.join(timeout=2)

    def summary(self):
        sms, maxes, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        lo, hi = getattr(self, "window", (0.0, float("inf")))
        for stamp, line in self.lines:
            if not (lo - 0.05 <= stamp <= hi + 0.25):  # output lags the sample slightly
                continue
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


# ---------------------------------------------------------------------------
# CPU reference (oracle) timing
# ---------------------------------------------------------------------------
class CpuSample:
    """The oracle on the bounded CPU sample of a workload (all host threads).

    The sample's inputs are copied to the host once (compact per-query
    copies, identical arithmetic); ``run()`` times one pass of the oracle
    over the sample and returns the seconds scaled to a full call."""

    def __init__(self, data, shape):
        from oracle import sparse_mla as oracle  # checker/baseline only

        self.oracle = oracle
        torch.set_num_threads(os.cpu_count() or 1)
        b, s, h, _, _ = shape
        self.total = b * s
        self.rows = min(self.total, CPU_SAMPLE_QUERIES)
        chunk = 16 if h >= 64 else 128
        self.chunks = [compact_for_oracle(data, list(range(r0, min(self.rows, r0 + chunk))))
                       for r0 in range(0, self.rows, chunk)]
        self.threads = torch.get_num_threads()

    def run(self):
        t0 = time.perf_counter()
        for compact in self.chunks:
            self.oracle.reference_forward(*compact)
        return (time.perf_counter() - t0) * self.total / self.rows

    def warm(self, seconds=2.0):
        """Untimed passes until the host threads reach their steady state."""
        end = time.perf_counter() + seconds
        self.run()
        while time.perf_counter() < end:
            self.run()

    def measure(self, seconds):
        """Median of full-call times over passes that fill at least `seconds`
        (at least one pass); returns (median seconds per call, passes)."""
        per_call, spent = [], 0.0
        while spent < seconds or not per_call:
            t0 = time.perf_counter()
            per_call.append(self.run())
            spent += time.perf_counter() - t0
        return statistics.median(per_call), len(per_call)

    def describe(self, passes):
        return (f"first {self.rows} of {self.total} queries ({100.0 * self.rows / self.total:.2f} %) per pass, "
                f"median of {passes} timed pass(es) after ~2 s of untimed passes; FP32 torch oracle of "
                f"tools/review.py:123-145 (HF32/TF32 off), scaled to a full call")


# ---------------------------------------------------------------------------
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def run_reference(args, shape):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    data = make_inputs_for(args, shape, dev)
    b, s, h, length, k = shape
    sample = CpuSample(data, shape)
    data = None
    sample.warm()
    # each step: the median over passes that fill >= 0.3 s (one pass when longer)
    per_call, passes = [], 0
    for i in range(args.warmup + args.steps):
        t, n = sample.measure(0.3)
        if i >= args.warmup:
            per_call.append(t)
            passes += n
    us = statistics.median(per_call) * 1e6
    threads = sample.threads
    line = {
        "impl": "reference", "metric": METRIC, "value": us, "unit": "us/call", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": us / 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, "B": b, "SQ": s, "H": h, "L": length, "TOPK": k,
                   "index_variant": args.variant, "seed": SEED},
        "cpu_baseline": {"value": us, "unit": "us/call", "cores": threads, "kind": "port",
                         "sample": sample.describe(passes) + "; per step the median over >= 0.3 s of passes, "
                                   "the line's value the median over steps"},
        "e2e": {"value": us, "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(CONFIGS))
    ap.add_argument("--shape", default=None,
                    help="B,SQ,H,L,TOPK override (a reduced case for profiling; workload 'custom')")
    ap.add_argument("--variant", default="uniform", choices=("uniform", "peaked", "duplicates"))
    ap.add_argument("--inputs", default="device", choices=("device", "reference"),
                    help="draw the inputs on the device (default) or in the reference's generator order on the CPU")
    ap.add_argument("--tuning", default=None,
                    help="bm,bn,split[,pv_cols] launch entry instead of the shape-keyed default "
                         "(selects a kernel family, e.g. 128,32,1,256 for the split-V family)")
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--direct", action="store_true",
                    help="time direct launches of the prepared forward instead of CUDA-graph replay")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    shape = CONFIGS[args.config]
    if args.shape:
        shape = tuple(int(v) for v in args.shape.split(","))
        if len(shape) != 5:
            raise SystemExit("--shape needs B,SQ,H,L,TOPK")
        args.config = "custom"
    if args.impl == "reference":
        return run_reference(args, shape)

    import dsa_b200
    from dsa_b200 import _native, sharded

    world, rank, local = init_dist()
    device = torch.device("cuda", local)
    b, s, h, length, k = shape
    data = make_inputs_for(args, shape, device)
    lo, hi = sharded.shard_bounds(b * s, world, rank)
    pieces = sharded.shard_pieces(s, lo, hi)
    views = [(data[0][b0:b1, s0:s1], data[1][b0:b1], data[2][b0:b1, s0:s1], data[3][b0:b1],
              data[4][b0:b1, s0:s1]) for b0, b1, s0, s1 in pieces]
    lib = _native.load()
    # The timed step replays a CUDA graph of the prepared forward (checks and
    # allocations done once, as a serving loop does); `e2e` below goes through
    # dsa_b200.forward with host copies every step.
    tuning = None
    if args.tuning:
        f = [int(v) for v in args.tuning.split(",")]
        tuning = dsa_b200.Tuning(f[0], f[1], f[2], pv_cols=f[3] if len(f) > 3 else 512)
    plans = [dsa_b200.ForwardPlan(*v, config=tuning) for v in views]
    for pl in plans:
        pl.run()
    torch.cuda.synchronize()
    kernels_per_step = sum(pl.kernels for pl in plans)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for pl in plans:
            pl.run()

    def step():
        if args.direct:
            for pl in plans:
                pl.run()
        else:
            graph.replay()
        return plans[-1].outputs, kernels_per_step

    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches_total = 0
    # a timed region of a few milliseconds (decode) fits between two 20 ms
    # clock samples: the same steps then also run untimed for ~60 ms just
    # before it, inside the sampled window, so the clock record covers this
    # load. Longer regions (prefill) are sampled as they are: extra load
    # before them would only push the GPU into its power cap earlier.
    t0 = time.perf_counter()
    step()
    torch.cuda.synchronize()
    step_s = max(time.perf_counter() - t0, 1e-5)
    load_steps = 0 if step_s * args.steps >= 0.02 else int(0.06 / step_s)
    with ClockSampler(local) as clocks:
        time.sleep(0.3)  # let nvidia-smi start sampling before the timed region
        t_host0 = time.time()
        for i in range(load_steps):
            flush.fill_(float(i))
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()
        for i in range(args.steps):
            flush.fill_(float(i))  # evict L2 between timed iterations (outside the events)
            starts[i].record(stream)
            _, n = step()
            ends[i].record(stream)
            launches_total += n
        torch.cuda.synchronize()
        clocks.mark(t_host0, time.time())
    durations = [a.elapsed_time(e) for a, e in zip(starts, ends)]  # ms
    total_ms = sum(durations)
    rank_ms = [total_ms / args.steps]
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([total_ms], device=device, dtype=torch.float64)
        every = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(every, t)
        rank_ms = [float(x.item()) / args.steps for x in every]
        total_ms = max(float(x.item()) for x in every)
    ms_per_step = total_ms / args.steps

    graph = None  # release the captured graph before the end-to-end part
    # End-to-end through the public API: every step copies its inputs from
    # pinned host memory to the device, calls dsa_b200.forward and reads its
    # outputs back into pinned host memory. Steps are pipelined as a serving
    # loop runs them: inputs on one copy stream, the forward on the compute
    # stream, outputs on another copy stream (host->device and device->host
    # share the link in opposite directions), with two buffer sets; the value
    # is the steady-state time per step.
    e2e_steps = args.e2e_steps or max(1, min(args.steps, 5))
    # this rank's inputs: its query rows of q, q_rope and the indices, and
    # kv / k_rope of the batch rows those queries read
    host_in = [[t.cpu().pin_memory() for t in vw] for vw in views]
    n_buf = 2
    dev_in = [[[torch.empty_like(t, device=device) for t in hp] for hp in host_in] for _ in range(n_buf)]
    out_host = [None] * n_buf
    h2d_bytes = sum(t.numel() * t.element_size() for hp in host_in for t in hp)
    data = None
    views = None
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(n_buf)]   # buffer b's inputs are on the device
    ev_fwd = [torch.cuda.Event() for _ in range(n_buf)]  # buffer b's forward is done
    ev_out = [torch.cuda.Event() for _ in range(n_buf)]  # buffer b's outputs are on the host
    step_no = [0]

    def e2e_step():
        b = step_no[0] % n_buf
        step_no[0] += 1
        s_in.wait_event(ev_fwd[b])  # the forward that last read these inputs is done
        with torch.cuda.stream(s_in):
            for hp, dp in zip(host_in, dev_in[b]):
                for hsrc, ddst in zip(hp, dp):
                    ddst.copy_(hsrc, non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        outs = [dsa_b200.forward(*dp, config=tuning) for dp in dev_in[b]]
        ev_fwd[b].record(stream)
        if out_host[b] is None:
            out_host[b] = [[torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in o] for o in outs]
        s_out.wait_event(ev_fwd[b])
        s_out.wait_event(ev_out[b])  # this host buffer's previous read-back is done
        with torch.cuda.stream(s_out):
            for o, hdst in zip(outs, out_host[b]):
                for t, hd in zip(o, hdst):
                    t.record_stream(s_out)
                    hd.copy_(t, non_blocking=True)
            ev_out[b].record(s_out)

    def drain():
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)

    e2e_step()
    e2e_step()
    drain()
    torch.cuda.synchronize()
    d2h_bytes = sum(t.numel() * t.element_size() for o in out_host[0] for t in o)
    if world > 1:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    drain()
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev0.elapsed_time(ev1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    gathered, other, flops = algorithmic(shape)
    hbm_peak, tf_peak, peak_kind = load_peaks()
    us = ms_per_step * 1e3
    # Roofline of the dominant kernel (the main kernel; for split == 1 configs
    # it is the only launch per call, so the per-call events time it).
    rank_share = (hi - lo) / (b * s)
    per_launch_flops = flops * rank_share
    per_launch_bytes = gathered * rank_share
    # Decode shapes are measured on gathered bytes against HBM, prefill shapes
    # (many queries per call) on FLOPs against the BF16 tensor peak.
    if s >= 64 or (args.config.startswith("prefill")):
        bound, achieved, peak, unit = "tensor", per_launch_flops / (ms_per_step * 1e-3) / 1e12, tf_peak, "TFLOP/s"
    else:
        bound, achieved, peak, unit = "hbm", per_launch_bytes / (ms_per_step * 1e-3) / 1e9, hbm_peak, "GB/s"
    line = {
        "metric": METRIC,
        "value": us,
        "unit": "us/call",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) BF16 q/kv/q_rope/k_rope, int32 top-k indices "
                + (f"({args.variant}), generated on the device" if args.inputs == "device" else
                   "(uniform), drawn in the reference's generator order (tools/review.py:35-61) on the CPU"),
        "config": {"workload": args.config, "B": b, "SQ": s, "H": h, "L": length, "TOPK": k,
                   "index_variant": args.variant, "seed": SEED, "inputs": args.inputs,
                   "parallelism": f"query-shard x{world}, kv replicated",
                   "l2": "flushed between timed iterations (256 MiB write outside the events)",
                   "timed": ("direct launches of ForwardPlan.run" if args.direct
                             else "CUDA-graph replay of ForwardPlan.run (one graph per step)"),
                   "launch": {"family": int(plans[0].launch.family), "split": int(plans[0].launch.split)}},
        "calls_per_s": 1e6 / us,
        "tflops": flops / (us * 1e-6) / 1e12,
        "gathered_gbs": gathered / (us * 1e-6) / 1e9,
        "step_ms": [round(d, 4) for d in durations],
        "step_ms_p10_p50_p90": [statistics.quantiles(durations, n=10)[0] if len(durations) > 1 else durations[0],
                                statistics.median(durations),
                                statistics.quantiles(durations, n=10)[-1] if len(durations) > 1 else durations[0]],
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json burst)",
                     "traffic": traffic_bytes(args.config, args.variant, bool(args.shape or args.tuning), hi - lo),
                     "traffic_source": "ncu capture of timed-loop launches of the default launch (uniform indices, after the L2 write flush), modelled per rank"},
        "e2e": {"value": e2e_ms * 1e3, "unit": "us/call", "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": d2h_bytes, "steps": e2e_steps,
                "mode": "pipelined: inputs in / forward / outputs out on three streams, two buffer sets"},
        "gpu_launches": launches_total,
        "clocks": dict(clocks.summary(), untimed_load_steps_in_window=load_steps),
    }
    if world > 1:
        line["ranks"] = {"n": world, "ms_per_step": rank_ms, "min_ms": min(rank_ms), "max_ms": max(rank_ms),
                         "argmax": max(range(world), key=lambda r: rank_ms[r]),
                         "queries": [sharded.shard_bounds(b * s, world, r)[1] - sharded.shard_bounds(b * s, world, r)[0]
                                     for r in range(world)]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the reference arm itself (bench.py --impl reference, same sample and
        # method), in a fresh child process after this process's GPU timing
        cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference", "--config",
               args.config if not args.shape else DEFAULT_CONFIG, "--variant", args.variant, "--steps", "5",
               "--warmup", "3", "--inputs", args.inputs] + (["--shape", args.shape] if args.shape else [])
        env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
        res = subprocess.run(cmd, capture_output=True, text=True, env=env)
        ref = None
        for ln in reversed(res.stdout.strip().splitlines()):
            try:
                ref = json.loads(ln)
                break
            except json.JSONDecodeError:
                continue
        if res.returncode == 0 and ref is not None and "cpu_baseline" in ref:
            cb = dict(ref["cpu_baseline"])
            cb["sample"] += "; measured by bench.py --impl reference (5 steps, 3 warm-up) in a child process of this run"
            line["cpu_baseline"] = cb
        else:
            line["cpu_baseline"] = {"value": None, "unit": "us/call", "cores": None, "kind": "port",
                                    "sample": f"reference arm failed (rc {res.returncode}): {res.stderr[-200:]}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
