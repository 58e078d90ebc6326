"""ncu profiling of the hot path (the reference's kernels/bench/profile.py, for a shared B200 pool).

    python llm-decode-kernels_b200/kernels/bench/profile.py command launches decode ours 2
    python llm-decode-kernels_b200/kernels/bench/profile.py command kernel w4a16_gemv gemv 151936 1536
    python llm-decode-kernels_b200/kernels/bench/profile.py run launches OUT.csv decode ours 2
    python llm-decode-kernels_b200/kernels/bench/profile.py summarize OUT.csv [--top 12]

The workloads are `profile_cases.py` cases (small and self-terminating). Every command carries
`--clock-control none` (the GPU's clocks are left alone). Two kinds of capture:
* `launches`: one metric (`gpu__time_duration.sum`, one replay pass) over a bounded number of
  launches - the launch list whose per-kernel shares go into the profile summaries;
* `kernel`: the full section set on one kernel (`-k`) and at most 3 launches (`-c`), for a small case.
`run` executes the workload once without ncu and profiles it only if that run exited 0 (a program
that faulted is never put under ncu). `summarize` turns the CSV of a launch list into the markdown
table of the summaries: per kernel its launches, total time and share.
"""

from __future__ import annotations

import argparse
import csv
import os
import subprocess
import sys
from collections import OrderedDict

CASES = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profile_cases.py")
MAX_FULL_LAUNCHES = 3


def ncu_command(kind: str, case: list[str], out: str, kernel: str | None = None, skip: int = 0,
                count: int | None = None) -> list[str]:
    """The ncu argv for one capture of `profile_cases.py <case...>`."""
    target = [sys.executable, CASES, *case]
    if kind == "launches":
        cmd = ["ncu", "--metrics", "gpu__time_duration.sum", "--clock-control", "none", "--csv", "--log-file", out]
        if skip:
            cmd += ["-s", str(skip)]
        cmd += ["-c", str(count if count is not None else 400)]
        return cmd + target
    if kind == "kernel":
        if not kernel:
            raise ValueError("a full-set capture needs a kernel filter (-k)")
        n = MAX_FULL_LAUNCHES if count is None else count
        if not 1 <= n <= MAX_FULL_LAUNCHES:
            raise ValueError(f"a full-set capture takes 1 to {MAX_FULL_LAUNCHES} launches")
        cmd = ["ncu", "--set", "full", "--clock-control", "none", "-k", f"regex:{kernel}", "-c", str(n), "-o", out]
        if skip:
            cmd[cmd.index("-c"):cmd.index("-c")] = ["-s", str(skip)]
        return cmd + target
    raise ValueError(f"unknown capture kind {kind!r} (launches or kernel)")


def run(kind: str, case: list[str], out: str, **kw) -> int:
    """Run the workload plainly; profile it only if that exited 0. Returns the exit status."""
    plain = subprocess.run([sys.executable, CASES, *case])
    if plain.returncode != 0:
        print(f"not profiled: the plain run exited {plain.returncode}", file=sys.stderr)
        return plain.returncode
    return subprocess.run(ncu_command(kind, case, out, **kw)).returncode


def _short(name: str) -> str:
    """Kernel name without its parameter list (template arguments kept)."""
    depth = 0
    for i, ch in enumerate(name):
        if ch == "<":
            depth += 1
        elif ch == ">":
            depth -= 1
        elif ch == "(" and depth == 0:
            name = name[:i]
            break
    return name.replace("void ", "", 1).strip()


def launch_summary(path: str) -> list[dict]:
    """Per kernel of an ncu launch-list CSV: launches, total and mean time (us), share of the total."""
    rows: OrderedDict[str, dict] = OrderedDict()
    with open(path, newline="") as f:
        lines = [ln for ln in f if ln.startswith('"')]
    for r in csv.DictReader(lines):
        if r.get("Metric Name") != "gpu__time_duration.sum":
            continue
        scale = {"ns": 1e-3, "us": 1.0, "usecond": 1.0, "nsecond": 1e-3, "ms": 1e3, "msecond": 1e3}.get(
            r.get("Metric Unit", "ns"), 1e-3)
        us = float(r["Metric Value"].replace(",", "")) * scale
        k = _short(r["Kernel Name"])
        e = rows.setdefault(k, {"kernel": k, "launches": 0, "total_us": 0.0})
        e["launches"] += 1
        e["total_us"] += us
    total = sum(e["total_us"] for e in rows.values()) or 1.0
    out = sorted(rows.values(), key=lambda e: -e["total_us"])
    for e in out:
        e["mean_us"] = e["total_us"] / e["launches"]
        e["share"] = e["total_us"] / total
    return out


def markdown(summary: list[dict], top: int | None = None) -> str:
    lines = ["| kernel | launches | total us | share |", "|---|---:|---:|---:|"]
    shown = summary[:top] if top else summary
    for e in shown:
        lines.append(f"| {e['kernel']} | {e['launches']} | {e['total_us']:.1f} | {100 * e['share']:.1f}% |")
    rest = summary[len(shown):]
    if rest:
        lines.append(f"| ({len(rest)} more kernels) | {sum(e['launches'] for e in rest)} | "
                     f"{sum(e['total_us'] for e in rest):.1f} | {100 * sum(e['share'] for e in rest):.1f}% |")
    lines.append(f"| **total** | {sum(e['launches'] for e in summary)} | {sum(e['total_us'] for e in summary):.1f} | |")
    return "\n".join(lines)


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("command", "run"):
        p = sub.add_parser(name)
        p.add_argument("kind", choices=["launches", "kernel"])
        if name == "run":
            p.add_argument("out")
        p.add_argument("case", nargs="+", help="[kernel regex for 'kernel'] profile_cases.py case and its args")
        p.add_argument("-s", "--skip", type=int, default=0)
        p.add_argument("-c", "--count", type=int, default=None)
    s = sub.add_parser("summarize")
    s.add_argument("csv")
    s.add_argument("--top", type=int, default=None)
    a = ap.parse_args(argv)
    if a.cmd == "summarize":
        print(markdown(launch_summary(a.csv), a.top))
        return 0
    kernel, case = (a.case[0], a.case[1:]) if a.kind == "kernel" else (None, a.case)
    out = getattr(a, "out", None) or ("launches.csv" if a.kind == "launches" else "prof")
    if a.cmd == "command":
        print(" ".join(ncu_command(a.kind, case, out, kernel=kernel, skip=a.skip, count=a.count)))
        return 0
    return run(a.kind, case, out, kernel=kernel, skip=a.skip, count=a.count)


if __name__ == "__main__":
    sys.exit(main())
