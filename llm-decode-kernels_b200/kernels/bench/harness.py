"""Kernel timing for the sweeps: CUDA-graph replays over rotating argument sets.

The measurement method is the reference's frozen one (kernels/bench/harness.py and
docs/DECISIONS.md:27-52 of the reference), so that "% of HBM peak" means the same number here:
copies of the rotated arguments until one pass over them is at least 4x the L2 size (every call
then reads DRAM, not L2), one CUDA graph holding one call per copy (no Python or launch-queue cost
in the timed region), replays until a sample lasts >= MIN_MS, and the median of MEASUREMENTS
samples. The code below is this package's own: a `_Timing` object owns the graph, its outputs and
the calibration, and `capture` is the one place graphs are made.
"""

from __future__ import annotations

import contextlib
import gc
import statistics
from collections.abc import Callable

import torch
from torch.utils import _pytree

WARMUP_CALLS = 3
MEASUREMENTS = 7
MIN_MS = 50.0
MEMORY_BUDGET = 3 * 1024**3  # bytes of rotating copies per case
MAX_COPIES = 512
L2_MULTIPLE = 4


def tensor_bytes(obj) -> int:
    """Bytes of every tensor inside `obj` (nested lists, tuples and dicts)."""
    return sum(t.numel() * t.element_size() for t in _pytree.tree_leaves(obj) if isinstance(t, torch.Tensor))


def n_copies(bytes_per_set: int, l2_mb: float) -> int:
    """How many argument sets make one pass at least L2_MULTIPLE x L2, bounded below by 2 and above
    by MAX_COPIES and by what fits in MEMORY_BUDGET."""
    per_set = max(int(bytes_per_set), 1)
    target = L2_MULTIPLE * l2_mb * 2**20
    needed = -(-int(target) // per_set)  # ceiling division
    fits = max(MEMORY_BUDGET // per_set, 2)
    return int(max(2, min(needed, fits, MAX_COPIES)))


@contextlib.contextmanager
def _collector_paused():
    """Python's garbage collector off (after one full collection): a CUDA object freed by the GC in
    the middle of a capture invalidates it."""
    gc.collect()
    was_on = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was_on:
            gc.enable()


def capture(body: Callable, retries: int = 1):
    """(graph, body's return value) for `body()` captured into a new CUDA graph in thread-local
    capture mode; a failed capture is retried `retries` more times before its error is raised."""
    attempts = retries + 1
    for attempt in range(attempts):
        graph = torch.cuda.CUDAGraph()
        try:
            with _collector_paused(), torch.cuda.graph(graph, capture_error_mode="thread_local"):
                result = body()
        except Exception:
            torch.cuda.synchronize()
            if attempt + 1 == attempts:
                raise
            continue
        return graph, result
    raise AssertionError("unreachable")


def _elapsed_ms(run: Callable[[], None]) -> float:
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    run()
    t1.record()
    t1.synchronize()
    return t0.elapsed_time(t1)


class _Timing:
    """One graph of `fn` over every argument set; the outputs stay referenced by the object so that
    each call writes fresh memory."""

    def __init__(self, fn: Callable, sets: list):
        self.calls = len(sets)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # first calls: library loads, kernel choices, allocations
            for args in sets[:WARMUP_CALLS]:
                fn(*args)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph, self.outputs = capture(lambda: [fn(*args) for args in sets])
        self.graph.replay()  # first replay uploads the graph
        torch.cuda.synchronize()

    def replays_for(self, ms: float) -> int:
        one = max(_elapsed_ms(self.graph.replay), 1e-3)
        return max(1, int(-(-ms // one)))

    def sample_ms_per_call(self, replays: int) -> float:
        def run():
            for _ in range(replays):
                self.graph.replay()

        return _elapsed_ms(run) / (replays * self.calls)

    def close(self):
        del self.graph, self.outputs


def time_graph(fn: Callable, sets: list) -> float:
    """Median milliseconds per call of `fn(*args)` over the argument sets, all calls in one graph."""
    timing = _Timing(fn, sets)
    try:
        replays = timing.replays_for(MIN_MS)
        return statistics.median(timing.sample_ms_per_call(replays) for _ in range(MEASUREMENTS))
    finally:
        timing.close()


def time_rotating(fn: Callable, args: tuple, rotate: tuple, max_copies: int = MAX_COPIES) -> float:
    """Graph time of fn(*args) with the tensors at positions `rotate` copied (n_copies of them, at most
    `max_copies`; the L2 size is read from the current device). Sets of under ~1 MB stay below 4x L2
    at 512 copies, as in the reference."""
    l2_mb = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size / 2**20
    rotated = set(rotate)
    copies = min(n_copies(sum(tensor_bytes(args[i]) for i in rotated), l2_mb), max_copies)

    def fresh_set():
        return tuple(a.clone() if i in rotated else a for i, a in enumerate(args))

    return time_graph(fn, [args, *(fresh_set() for _ in range(copies - 1))])


def metrics(ms: float, bytes_moved: int, flops: int, peak_gbps: float, peak_tflops: float) -> dict:
    """Achieved bandwidth and throughput of one timed call against the given peaks (the reference's
    result fields: gbps, pct_peak_bw, tflops, pct_peak_flops, intensity)."""
    seconds = ms / 1e3
    gbps = bytes_moved / seconds / 1e9
    out = {"gbps": gbps, "pct_peak_bw": 100.0 * gbps / peak_gbps, "tflops": 0.0, "pct_peak_flops": 0.0,
           "intensity": 0.0}
    if flops:
        tflops = flops / seconds / 1e12
        out.update(tflops=tflops, pct_peak_flops=100.0 * tflops / peak_tflops, intensity=flops / bytes_moved)
    return out
