"""Layer sweeps of the decode hot path with the reference's sweep policy.

    python llm-decode-kernels_b200/kernels/bench/sweep.py [--kernels copy,rmsnorm,swiglu,w4a16]
                                                          [--sweeps 3] [--quick] [--out FILE]
                                                          [--checkpoint FILE.jsonl]

Cases (the benchmark configurations of the hot path):
* w4a16: every Qwen2.5-1.5B linear shape at M in {1, 4, 16}, for our W4A16 matmul ("ours"), our
  FP8 e4m3 weight-only matmul ("fp8") and cuBLAS fp16 `F.linear` ("fp16", 4x the weight bytes);
* rmsnorm: [M, 1536] with and without the residual add, M in {1, 16, 2048};
* swiglu: [M, 2 x 8960] gate|up halves, M in {1, 16, 2048};
* copy: a 128 MiB device-to-device copy, the practical bandwidth ceiling.

Each case is timed by `harness.time_rotating`: CUDA graph, every input copied until the working
set is >= 4x L2, >= 50 ms of replays, median of 7. The whole sweep then runs `sweeps` times and
each case reports the median over sweeps with min and max, flagging spreads over 10% (reference
kernels/bench/sweep.py:206-233, docs/DECISIONS.md:27-52). Algorithmic bytes follow the reference:
matmuls M*K*2 + M*N*2 + weight bytes, RMSNorm `rmsnorm_bytes`, SwiGLU `swiglu_bytes`.

Checkpoints (`--checkpoint`) are a local JSONL file of finished rows. The reference's Modal volume,
torch.compile and torchao baselines are not part of the decode hot path and are left out.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

if __name__ == "__main__":
    sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..")))

from kernels import config  # noqa: E402

KERNELS = ("copy", "rmsnorm", "swiglu", "w4a16")
DECODE_M = (1, 4, 16)
NORM_M = (1, 16, 2048)
HIDDEN = 1536
INTER = 8960
COPY_ELEMS = 64 * 2**20
W4_IMPLS = ("ours", "fp8", "fp16")


def case_specs(kernels=KERNELS, quick: bool = False) -> list[dict]:
    """The (kernel, impl, shape) of every case, in sweep order; no device work."""
    specs = []
    shapes = config.QWEN15_SHAPES[:2] if quick else config.QWEN15_SHAPES
    for k in kernels:
        if k == "copy":
            specs.append({"kernel": "copy", "impl": "torch", "shape": {"elems": COPY_ELEMS}})
        elif k == "rmsnorm":
            for residual in (True, False):
                for M in NORM_M:
                    specs.append({"kernel": "rmsnorm", "impl": "ours", "shape": {"M": M, "N": HIDDEN, "residual": residual}})
        elif k == "swiglu":
            for M in NORM_M:
                specs.append({"kernel": "swiglu", "impl": "ours", "shape": {"M": M, "I": INTER}})
        elif k == "w4a16":
            for label, N, K in shapes:
                for M in DECODE_M:
                    for impl in W4_IMPLS:
                        specs.append({"kernel": "w4a16", "impl": impl, "shape": {"layer": label, "M": M, "N": N, "K": K}})
        else:
            raise ValueError(f"unknown kernel {k!r}; choose from {KERNELS}")
    return specs


def bytes_and_flops(spec: dict) -> tuple[int, int]:
    """Algorithmic bytes (each input read once, each output written once) and flops of a case."""
    from kernels.fp8 import fp8_bytes
    from kernels.quant import weight_bytes
    from kernels.rmsnorm import rmsnorm_bytes
    from kernels.swiglu import swiglu_bytes

    s, k = spec["shape"], spec["kernel"]
    if k == "copy":
        return 2 * s["elems"] * 2, 0
    if k == "rmsnorm":
        return rmsnorm_bytes(s["M"], s["N"], s["residual"]), 0
    if k == "swiglu":
        return swiglu_bytes(s["M"], s["I"]), 0
    M, N, K = s["M"], s["N"], s["K"]
    act = M * K * 2 + M * N * 2
    weights = {"ours": weight_bytes(N, K), "fp8": fp8_bytes(N, K), "fp16": N * K * 2}[spec["impl"]]
    return act + weights, 2 * M * N * K


class _Weights:
    """Each layer shape's weights in the three formats, made once and shared by all sweeps."""

    def __init__(self):
        self.cache = {}

    def get(self, N: int, K: int):
        if (N, K) not in self.cache:
            import torch

            from kernels.fp8 import quantize_fp8
            from kernels.quant import quantize_rtn

            g = torch.Generator(device="cuda").manual_seed(0)
            w16 = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
            self.cache[(N, K)] = {"fp16": w16, "ours": quantize_rtn(w16, config.GROUP_SIZE), "fp8": quantize_fp8(w16)}
        return self.cache[(N, K)]


def time_case(spec: dict, weights: _Weights) -> float:
    """Milliseconds per call of one case (harness.time_rotating, every input rotated)."""
    import torch
    import torch.nn.functional as F

    from kernels.bench.harness import time_rotating

    s, k, impl = spec["shape"], spec["kernel"], spec["impl"]
    g = torch.Generator(device="cuda").manual_seed(1)

    def randn(*shape):
        return torch.randn(*shape, device="cuda", generator=g).half()

    if k == "copy":
        src = randn(s["elems"])
        return time_rotating(lambda a, b: b.copy_(a), (src, torch.empty_like(src)), rotate=(0, 1))
    if k == "rmsnorm":
        from kernels.rmsnorm import rmsnorm

        M, N = s["M"], s["N"]
        w = (1 + 0.05 * randn(N).float()).half()
        if s["residual"]:
            return time_rotating(lambda x, r: rmsnorm(x, w, 1e-6, r), (randn(M, N), randn(M, N)), rotate=(0, 1))
        return time_rotating(lambda x: rmsnorm(x, w, 1e-6), (randn(M, N),), rotate=(0,))
    if k == "swiglu":
        from kernels.swiglu import swiglu_fused

        return time_rotating(swiglu_fused, (randn(s["M"], 2 * s["I"]),), rotate=(0,))
    M, N, K = s["M"], s["N"], s["K"]
    x = randn(M, K)
    wt = weights.get(N, K)
    if impl == "ours":
        from kernels.w4a16 import w4a16_matmul

        qw, sc, z = wt["ours"]
        return time_rotating(lambda xx, q, ss, zz: w4a16_matmul(xx, q, ss, zz), (x, qw, sc, z), rotate=(0, 1, 2, 3))
    if impl == "fp8":
        from kernels.fp8 import w8a16_matmul

        wq, s8 = wt["fp8"]
        return time_rotating(lambda xx, q, ss: w8a16_matmul(xx, q, ss), (x, wq, s8), rotate=(0, 1, 2))
    return time_rotating(F.linear, (x, wt["fp16"]), rotate=(0, 1))


def _row_key(row: dict) -> str:
    return json.dumps([row["sweep"], row["kernel"], row["impl"], row["shape"]], sort_keys=True)


def run(kernels=KERNELS, sweeps: int = 3, quick: bool = False, log=None, checkpoint: str | None = None) -> list[dict]:
    """Raw rows: one per (sweep, case), {"ms": ...} or {"error": ...} (a failing case is recorded
    and the sweep goes on). With `checkpoint`, every finished row is appended to that JSONL file as
    it completes, and rows already in it are reused instead of measured again, so an interrupted
    sweep resumes where it stopped (the reference's resumable sweeps, kernels/bench/sweep.py:3-4)."""
    specs = case_specs(kernels, quick)
    done = {}
    if checkpoint and os.path.exists(checkpoint):
        with open(checkpoint) as f:
            for line in f:
                line = line.strip()
                if line:
                    r = json.loads(line)
                    done[_row_key(r)] = r
    sink = open(checkpoint, "a") if checkpoint else None
    weights = _Weights()
    rows = []
    try:
        for sweep in range(sweeps):
            for spec in specs:
                row = {**spec, "sweep": sweep}
                if _row_key(row) in done:
                    rows.append(done[_row_key(row)])
                    continue
                try:
                    row["ms"] = time_case(spec, weights)
                except Exception as e:  # recorded, not hidden
                    row["error"] = f"{type(e).__name__}: {e}"[:300]
                rows.append(row)
                if sink is not None:
                    sink.write(json.dumps(row) + "\n")
                    sink.flush()
                if log is not None:
                    log(row)
    finally:
        if sink is not None:
            sink.close()
    return rows


def aggregate(rows: list[dict], peak_gbs: float, peak_tflops: float) -> list[dict]:
    """Median over sweeps per (kernel, impl, shape), with min, max, spread and the >10% flag;
    GB/s and % of the bandwidth peak from the algorithmic bytes, TFLOP/s for matmuls."""
    groups: dict[str, list[dict]] = {}
    order = []
    for r in rows:
        key = json.dumps([r["kernel"], r["impl"], r["shape"]], sort_keys=True)
        if key not in groups:
            groups[key] = []
            order.append(key)
        groups[key].append(r)
    out = []
    for key in order:
        rs = groups[key]
        ok = [r["ms"] for r in rs if "ms" in r]
        first = rs[0]
        row = {"kernel": first["kernel"], "impl": first["impl"], "shape": first["shape"], "sweeps": len(ok)}
        errors = [r["error"] for r in rs if "error" in r]
        if errors:
            row["error"] = errors[0]
        if ok:
            med = statistics.median(ok)
            byts, flops = bytes_and_flops(first)
            spread = 100.0 * (max(ok) - min(ok)) / med
            row.update({"us": round(med * 1e3, 3), "us_min": round(min(ok) * 1e3, 3), "us_max": round(max(ok) * 1e3, 3),
                        "spread_pct": round(spread, 1), "flag_spread": spread > 10.0,
                        "gbs": round(byts / (med * 1e-3) / 1e9, 1),
                        "pct_peak": round(100.0 * byts / (med * 1e-3) / 1e9 / peak_gbs, 1)})
            if flops:
                tf = flops / (med * 1e-3) / 1e12
                row.update({"tflops": round(tf, 2), "pct_peak_tflops": round(100.0 * tf / peak_tflops, 2)})
        out.append(row)
    return out


def compact(agg: list[dict]) -> dict:
    """One short entry per case for a benchmark line: 'kernel/impl/shape' -> us, % of peak, spread."""
    out = {}
    for r in agg:
        s = r["shape"]
        if r["kernel"] == "w4a16":
            name = f"w4a16/{r['impl']}/{s['layer']}/M{s['M']}"
        elif r["kernel"] == "rmsnorm":
            name = f"rmsnorm/M{s['M']}" + ("/residual" if s["residual"] else "")
        elif r["kernel"] == "swiglu":
            name = f"swiglu/M{s['M']}"
        else:
            name = r["kernel"]
        out[name] = ({"us": r["us"], "pct_peak": r["pct_peak"], "spread_pct": r["spread_pct"]} if "us" in r
                     else {"error": r.get("error", "no timing")})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernels", default=",".join(KERNELS))
    ap.add_argument("--sweeps", type=int, default=3)
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--out", default=None, help="write raw rows and the aggregate as JSON")
    ap.add_argument("--checkpoint", default=None, help="JSONL of finished rows: appended to, and reused on a rerun")
    args = ap.parse_args()
    pk = config.peaks()
    kernels = [k for k in args.kernels.split(",") if k]
    rows = run(kernels, args.sweeps, args.quick, log=lambda r: print(json.dumps(r), flush=True),
               checkpoint=args.checkpoint)
    agg = aggregate(rows, pk["hbm_gbs"], pk["bf16_tflops"])
    for r in agg:
        print(json.dumps(r), flush=True)
    if args.out:
        with open(args.out, "w") as f:
            json.dump({"peaks": pk, "rows": rows, "aggregate": agg}, f)


if __name__ == "__main__":
    main()
