"""CUDA-graph timing with rotating buffers (the reference's frozen method, kernels/bench/harness.py
and docs/DECISIONS.md:27-52): input copies until the working set is >= 4x L2 so every call reads
DRAM, one CUDA graph of one call per copy, replays for >= 50 ms, median of 7."""

from __future__ import annotations

import gc
import math
import statistics
from collections.abc import Callable

import torch

WARMUP_CALLS = 3
MEASUREMENTS = 7
MIN_MS = 50.0
MEMORY_BUDGET = 3 * 1024**3  # bytes of rotating copies per case


def tensor_bytes(obj) -> int:
    if isinstance(obj, torch.Tensor):
        return obj.numel() * obj.element_size()
    if isinstance(obj, (list, tuple)):
        return sum(tensor_bytes(o) for o in obj)
    if isinstance(obj, dict):
        return sum(tensor_bytes(o) for o in obj.values())
    return 0


def n_copies(bytes_per_set: int, l2_mb: float) -> int:
    want = math.ceil(4 * l2_mb * 2**20 / max(bytes_per_set, 1))
    cap = max(2, MEMORY_BUDGET // max(bytes_per_set, 1))
    return int(min(max(want, 2), cap, 512))


def capture(body: Callable, retries: int = 1):
    """Capture `body()` into a CUDA graph and return (graph, body's result); GC off during capture,
    thread-local capture mode, one retry (reference harness.py:46-67)."""
    last = None
    for _ in range(retries + 1):
        graph = torch.cuda.CUDAGraph()
        gc.collect()
        gc.disable()
        try:
            with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                out = body()
            return graph, out
        except Exception as e:  # torch.AcceleratorError and friends
            last = e
            torch.cuda.synchronize()
        finally:
            gc.enable()
    raise last


def time_graph(fn: Callable, sets: list) -> float:
    """Median ms per call with all calls captured in one CUDA graph; every call keeps its own output
    alive so writes do not stay in L2 (reference harness.py:70-103)."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for args in sets[:WARMUP_CALLS]:
            fn(*args)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph, outs = capture(lambda: [fn(*args) for args in sets])
    graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    graph.replay()
    end.record()
    torch.cuda.synchronize()
    replays = max(1, math.ceil(MIN_MS / max(start.elapsed_time(end), 1e-3)))
    samples = []
    for _ in range(MEASUREMENTS):
        start.record()
        for _ in range(replays):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
        samples.append(start.elapsed_time(end) / (replays * len(sets)))
    del graph, outs
    return statistics.median(samples)


def time_rotating(fn: Callable, args: tuple, rotate: tuple, max_copies: int = 512) -> float:
    """Graph time of fn(*args) with the tensors at positions `rotate` copied until the working set
    exceeds 4x L2 (read from the device), within `n_copies`' limits (at most 512 copies and 3 GiB,
    at least 2: the reference's measure(), kernels/bench/harness.py:144-160). Sets of under ~1 MB
    (RMSNorm or SwiGLU of a few rows) stay below 4x L2 at 512 copies, as in the reference."""
    l2_mb = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size / 2**20
    nbytes = sum(tensor_bytes(args[i]) for i in rotate)
    copies = min(n_copies(nbytes, l2_mb), max_copies)
    sets = [args] + [tuple(a.clone() if i in rotate else a for i, a in enumerate(args)) for _ in range(copies - 1)]
    return time_graph(fn, sets)


def metrics(ms: float, bytes_moved: int, flops: int, peak_gbps: float, peak_tflops: float) -> dict:
    s = ms * 1e-3
    gbps = bytes_moved / s / 1e9
    tflops = flops / s / 1e12 if flops else 0.0
    return {"gbps": gbps, "pct_peak_bw": 100 * gbps / peak_gbps, "tflops": tflops,
            "pct_peak_flops": 100 * tflops / peak_tflops if flops else 0.0,
            "intensity": flops / bytes_moved if flops else 0.0}
