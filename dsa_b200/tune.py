"""Measure the launch entries that apply to a shape and print a SELECTED table.

The reference tunes one launch entry per validated shape and keeps the
winners in ``SELECTED`` (dsa/config.py:42-62). This is the same step for
B200: for every named shape of ``config.CASE_SHAPES`` (or the ones given)
it times the library's shape-only heuristic and every candidate entry that
``dsa_check_launch`` accepts for the shape, on seeded random inputs with the
L2 flushed between calls (CUDA events on the current stream, median of the
repetitions), and prints the entries that beat the heuristic by more than
``--margin``.

    python -m dsa_b200.tune [--names decode_b8,prefill_q64] [--reps 20] [--margin 0.03]

Timing only: parity of every family is the test suite's job.
"""
from __future__ import annotations

import argparse
import statistics

import torch

from . import api, config
from .config import Tuning

_FLUSH_BYTES = 256 << 20  # > the 126 MB L2


def candidates(shape):
    """Launch entries to try for ``shape`` (unsupported ones are skipped)."""
    _, _, heads, _, topk = shape
    tiles32 = (topk + 31) // 32
    out = []
    if heads == 128:
        out.append(Tuning(128, 32, 1, pv_cols=512))
        out += [Tuning(128, 32, s, pv_cols=512) for s in (2, 4)]
        out += [Tuning(128, 32, s, pv_cols=256) for s in (1, 2, 4, 8, 16) if s <= tiles32]
    else:
        out += [Tuning(16, 32, s) for s in (1, 2, 4, 8) if s <= tiles32]
        out.append(Tuning(16, 32, 1, pv_cols=128))  # union launch of the pair family
        out += [Tuning(16, 64, s, pv_cols=128) for s in (1, 2, 4)]
        out += [Tuning(16, 64, s) for s in (1, 2, 4)]
    return out


def _inputs(shape, seed, device):
    b, s, h, length, topk = shape
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    q = torch.randn((b, s, h, 512), generator=g, device=device).to(torch.bfloat16)
    kv = torch.randn((b, length, 1, 512), generator=g, device=device).to(torch.bfloat16)
    q_rope = torch.randn((b, s, h, 64), generator=g, device=device).to(torch.bfloat16)
    k_rope = torch.randn((b, length, 1, 64), generator=g, device=device).to(torch.bfloat16)
    ids = torch.randint(0, length, (b, s, 1, topk), generator=g, device=device, dtype=torch.int32)
    return q, kv, q_rope, k_rope, ids


def time_entry(data, tuning, reps, flush):
    """Median µs per call of ``ForwardPlan.run`` with ``tuning`` (None: the
    library heuristic), or None when the entry does not apply."""
    try:
        plan = api.ForwardPlan(*data, config=tuning)
    except ValueError:
        return None
    for _ in range(3):
        plan.run()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    times = []
    for i in range(reps):
        flush.fill_(float(i))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        plan.run()
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    return statistics.median(times)


def tune(names, reps=20, margin=0.03, seed=20261103, verbose=False):
    """{name: (heuristic µs, best Tuning or None, best µs)} for ``names``."""
    saved = dict(config.SELECTED)
    config.SELECTED.clear()
    config._rebuild_index()
    api._default_cache.clear()
    device = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    results = {}
    try:
        for name in names:
            shape = config.CASE_SHAPES[name]
            data = _inputs(shape, seed, device)
            base = time_entry(data, None, reps, flush)
            best, best_us = None, base
            for t in candidates(shape):
                us = time_entry(data, t, reps, flush)
                if verbose:
                    print(f"    {t}: {'not applicable' if us is None else f'{us:.1f} us'}", flush=True)
                if us is not None and us < best_us * (1.0 - margin):
                    best, best_us = t, us
            results[name] = (base, best, best_us)
            print(f"{name:22s} {shape}: heuristic {base:10.1f} us; best "
                  f"{'heuristic' if best is None else best} {best_us:10.1f} us", flush=True)
            del data
    finally:
        config.SELECTED.clear()
        config.SELECTED.update(saved)
        config._rebuild_index()
        api._default_cache.clear()
    return results


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--names", default=None, help="comma-separated CASE_SHAPES names (default: all)")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--margin", type=float, default=0.03)
    ap.add_argument("--verbose", action="store_true", help="print every candidate's time")
    args = ap.parse_args()
    names = args.names.split(",") if args.names else list(config.CASE_SHAPES)
    results = tune(names, args.reps, args.margin, verbose=args.verbose)
    print("SELECTED = {")
    for name, (_, best, _) in results.items():
        if best is not None:
            print(f"    {name!r}: {best!r},")
    print("}")


if __name__ == "__main__":
    main()
