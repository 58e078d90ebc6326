#!/usr/bin/env python
"""Benchmark of the decode hot path: Qwen2.5-1.5B-architecture batch-1 decode tok/s under CUDA
graphs with libdecodek's W4A16 kernels, plus the W4A16 GEMV roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]

One process per GPU (torchrun for N > 1). The batch-1 1.5B path does not shard (each GPU holds the
whole model), so N GPUs run N independent replicas: weak scaling, `value` = tokens of all ranks /
the slowest rank's time. A "step" is one decode token (one graph replay) per replica.

`--impl reference` times the reference's CPU path for the same config on the host cores: the
oracle's restatement of the runner with dequantize-then-matmul fp32 linears
(kernels/reference.py:39-45), a bounded number of decode steps at the same cache length.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (str(ROOT), str(ROOT / "llm-decode-kernels_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402

METRIC = "Qwen2.5-1.5B decode tok/s batch 1"
PROMPT = 512
MAX_LEN = 2048


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--backend", default="ours", help="runner backend of our arm (ours, ours_lm, ours_fp8)")
    ap.add_argument("--no-extras", action="store_true", help="skip fp16 baseline, GEMV sweep and CPU baseline")
    ap.add_argument("--l2-prefetch", action="store_true",
                    help="runner with cross-launch L2 prefetch of the next projections' weights")
    ap.add_argument("--tp7b", choices=["auto", "on", "off"], default="auto",
                    help="Qwen2.5-7B tensor-parallel decode over the N ranks (BASELINE configs[4], TP=1 at N=1); "
                         "auto = on unless --no-extras")
    ap.add_argument("--fused-step", action="store_true",
                    help="run the decode step as the single fused decode-step kernel instead of the per-op kernels")
    ap.add_argument("--tp-batches", default="1,8,32", help="batch sizes of the 7B tensor-parallel decode")
    return ap.parse_args()


# ------------------------------------------------------------------------------ distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples during the timed region (clocks, power, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def env_info() -> dict:
    """GPU, driver, toolkit and library versions of this run (the reference's env_info,
    kernels/remote.py:15-52)."""
    import platform

    out = {"torch": torch.__version__, "cuda_runtime": torch.version.cuda, "python": platform.python_version(),
           "host_cpus": os.cpu_count()}
    try:
        if torch.cuda.is_available():
            p = torch.cuda.get_device_properties(torch.cuda.current_device())
            out.update(gpu=p.name, capability=f"{p.major}.{p.minor}", sms=p.multi_processor_count,
                       memory_gib=round(p.total_memory / 2**30, 1))
        r = subprocess.run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"],
                           capture_output=True, text=True, timeout=10)
        if r.returncode == 0 and r.stdout.strip():
            out["driver"] = r.stdout.strip().splitlines()[0]
    except Exception as e:  # informational only
        out["env_error"] = f"{type(e).__name__}: {e}"[:200]
    return out


# ------------------------------------------------------------------------------ model
def build_model(batch: int, seed: int = 0):
    from kernels import config
    from kernels.e2e.model import random_qwen2

    model = random_qwen2(config.QWEN15, dtype=torch.float16, device="cuda", seed=seed)
    return model


def prompt_ids(vocab: int, batch: int, seed: int = 1, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(0, vocab, (batch, PROMPT), generator=g).to(device)


def time_decode(dec, ids, steps: int, warmup: int, world: int) -> float:
    """Seconds for `steps` graph replays after `warmup` untimed ones, bracketed by barrier + sync."""
    dec.prefill(ids)
    for _ in range(warmup):
        dec.graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        dec.graph.replay()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end) / 1e3


def step_bytes(runner, pos: float) -> float:
    """Algorithmic bytes of one greedy decode step at cache position `pos` (every weight once, the
    KV-cache rows 0..pos once): packed linears with scales, zeros and biases, the fp16 lm_head, the
    RMSNorm weights, the batch's embedding rows, K and V rows read (pos + 1 per sequence, kv head and
    layer) and written (one each), and the RoPE rows. Activations between ops stay on chip or in L2
    and are not counted."""
    B, L, H = runner.batch, len(runner.layers), runner.embed.shape[1]
    wb = runner.weight_bytes()
    kv_row = runner.head_dim * 2
    kv = 2 * L * B * runner.n_kv * kv_row * (pos + 1 + 1)
    norms = (2 * L + 1) * H * 2
    return wb["linear_layers"] + wb["lm_head_read"] + norms + B * H * 2 + kv + 2 * kv_row


def step_roofline(runner, sec_per_step: float, first_pos: int, steps: int, peak_gbs: float) -> dict:
    """The dominant kernel: the fused decode step (decode_step_kernel, one launch per token, the whole
    step). achieved = algorithmic bytes of a step (at the mean position of the timed steps) / the
    measured time per step (CUDA events around the timed graph replays, one launch each, so the
    launch-to-launch gap is counted against the kernel)."""
    pos = first_pos + (steps - 1) / 2
    byts = step_bytes(runner, pos)
    achieved = byts / sec_per_step / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4), "traffic": step_traffic(),
            "kernel": "decode_step_kernel (fused greedy decode step, 1 launch per token)",
            "bytes_per_launch": round(byts), "us_per_launch": round(sec_per_step * 1e6, 3),
            "mean_position": pos}


def step_traffic():
    """DRAM bytes per launch of the fused step from the committed ncu summary of the same workload."""
    f = ROOT / "profiles" / "decode_step_kernel_traffic.json"
    try:
        return json.loads(f.read_text())["dram_bytes_per_launch"]
    except Exception:
        return None


def parity_on_benchmark_model(model, ids, steps: int = 32) -> dict:
    """The north star's greedy-stream bar on the benchmark model itself: `steps` greedy tokens of the
    benchmarked per-op step (its layers and its lm_head + greedy-pick kernel) and of the fused step,
    each against the reference numerics (w4_ref: dequantize, cuBLAS fp16, SDPA), with the reference's
    parity figures (kernels/e2e/run.py:289-303)."""
    from kernels.e2e.model import QwenRunner, make_backend
    from kernels.e2e.run import greedy_parity
    from kernels.head import KernelHeadLogits
    from kernels.step import StepLogits

    out = {"vs": "w4_ref (reference numerics)", "steps": steps, "prompt": ids.shape[1]}
    ref = QwenRunner(model, make_backend("w4_ref"), max_len=MAX_LEN)
    for name, fused, view in (("per_op", False, KernelHeadLogits), ("fused_step", True, StepLogits)):
        ours = QwenRunner(model, make_backend("ours"), max_len=MAX_LEN, fused_step=fused)
        ref.k_cache.zero_()
        ref.v_cache.zero_()
        r = greedy_parity(view(ours), ref, ids[:1], steps=steps)
        del ours
        torch.cuda.empty_cache()
        tol = 5e-2 + 5e-2 * r["max_abs_ref_logit"]
        ok = r["max_abs_logit_diff"] <= tol and (r["first_divergence"] == steps or r["ref_margin_at_divergence"] <= 2 * tol)
        out[name] = {"max_abs_logit_diff": round(r["max_abs_logit_diff"], 5),
                     "max_abs_ref_logit": round(r["max_abs_ref_logit"], 3), "first_divergence": r["first_divergence"],
                     "ref_margin_at_divergence": r["ref_margin_at_divergence"], "tolerance": round(tol, 4),
                     "pass": bool(ok)}
    del ref
    torch.cuda.empty_cache()
    out["pass"] = all(out[k]["pass"] for k in ("per_op", "fused_step"))
    return out


def decode_variant(model, backend: str, batch: int, steps: int, warmup: int, fused: bool = False,
                   l2_prefetch: bool = False) -> dict:
    """tok/s of another configs[3] variant on the same model (same prompt method, graph decoder)."""
    from kernels.e2e.model import QwenRunner, make_backend
    from kernels.e2e.run import GraphDecoder

    runner = QwenRunner(model, make_backend(backend), max_len=MAX_LEN, batch=batch, fused_step=fused,
                        l2_prefetch=l2_prefetch)
    ids = prompt_ids(model.config.vocab_size, batch)
    dec = GraphDecoder(runner)
    dec.capture(ids)
    sec = time_decode(dec, ids, steps, warmup, 1)
    path = "fused step" if runner.step_kernel() is not None else "per-op kernels"
    del dec, runner
    torch.cuda.empty_cache()
    return {"backend": backend, "batch": batch, "path": path, "l2_prefetch": l2_prefetch,
            "tok_s": round(batch * steps / sec, 1), "ms_per_step": round(sec / steps * 1e3, 4)}


def gemv_roofline(runner, peak_gbs: float) -> dict:
    """The dominant kernel (W4A16 GEMV): one decode step's linears, issued exactly as the decode step
    issues them (per layer norm+qkv, o, norm+gate_up+SwiGLU, down; M = 1; the runner's L2 prefetch
    plan), captured back to back in one CUDA graph on the current stream and timed with CUDA events;
    achieved = algorithmic bytes of those launches / their time."""
    from kernels.bench.harness import capture
    from kernels.quant import weight_bytes

    be = runner.backend
    H = runner.embed.shape[1]
    x = torch.randn(1, 1, H, device="cuda", dtype=torch.float16)
    nq, hd = runner.n_heads, runner.head_dim
    a = torch.randn(1, 1, nq * hd, device="cuda", dtype=torch.float16)
    I = runner.layers[0].down.qweight.shape[0] * 8

    r = torch.randn(1, 1, H, device="cuda", dtype=torch.float16)

    split_sums = getattr(be, "partials", False) and runner.tp is None

    def chain():  # as QwenRunner._decode_layers issues them at one row (down_proj's partial sums included)
        parts, n = None, len(runner.layers)
        for i, L in enumerate(runner.layers):
            if parts is not None:
                be.norm_linear_partials(parts, runner.layers[i - 1].down.bias, L.ln1, runner.eps, r, L.qkv)
            else:
                be.norm_linear(x, L.ln1, runner.eps, r, L.qkv)
            be.linear(a, L.o)
            act, _ = be.norm_gate_up_act(x, L.ln2, runner.eps, r, L.gate_up)
            if split_sums and i + 1 < n:
                parts = be.linear_partials(act, L.down)
            else:
                be.linear(act, L.down)
                parts = None

    chain()
    torch.cuda.synchronize()
    graph, _ = capture(chain)
    graph.replay()
    torch.cuda.synchronize()
    reps = 20
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    sec = start.elapsed_time(end) / 1e3 / reps
    launches = 4 * len(runner.layers)
    byts = 0
    for L in runner.layers:
        for p, k_in, n_out in ((L.qkv, H, L.qkv.qweight.shape[1]), (L.o, nq * hd, H),
                               (L.gate_up, H, I), (L.down, I, H)):
            N = p.qweight.shape[1]
            K = p.qweight.shape[0] * 8
            byts += weight_bytes(N, K) + 2 * k_in + 2 * n_out + (2 * N if p.bias is not None else 0)
    del graph
    achieved = byts / launches / (sec / launches) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4), "traffic": traffic_per_launch(),
            "kernel": "w4a16_gemv_kernel (28 x {norm+qkv, o_proj, norm+gate_up+SwiGLU, down}, M=1)",
            "bytes_per_launch": round(byts / launches), "us_per_launch": round(sec / launches * 1e6, 3)}


def traffic_per_launch():
    """DRAM bytes per launch of the GEMV from the committed ncu summary of the same decode chain."""
    f = ROOT / "profiles" / "w4a16_gemv_decode_chain.json"
    try:
        return json.loads(f.read_text())["dram_bytes_per_launch"]
    except Exception:
        return None


def gemv_sweep(peak_gbs: float) -> dict:
    """W4A16 GEMV % of HBM peak at M = 1 on every Qwen2.5-1.5B linear shape, timed like the
    reference's harness (CUDA graph, rotating weight copies >= 4x L2)."""
    from kernels import config
    from kernels.bench.harness import time_rotating
    from kernels.quant import quantize_rtn, weight_bytes
    from kernels.w4a16 import w4a16_matmul

    out = {}
    cfg = {"STATIC_WEIGHTS": True}
    for label, N, K in config.QWEN15_SHAPES:
        w = (torch.randn(N, K, device="cuda") * 0.02).half()
        qw, s, z = quantize_rtn(w, 128)
        del w
        x = torch.randn(1, K, device="cuda", dtype=torch.float16)
        ms = time_rotating(lambda xx, q, ss, zz: w4a16_matmul(xx, q, ss, zz, config=cfg), (x, qw, s, z),
                           rotate=(1, 2, 3))
        byts = weight_bytes(N, K) + 2 * K + 2 * N
        gbs = byts / (ms * 1e-3) / 1e9
        out[label] = {"N": N, "K": K, "us": round(ms * 1e3, 2), "gbs": round(gbs), "pct_peak": round(100 * gbs / peak_gbs, 1)}
        del qw, s, z
        torch.cuda.empty_cache()
    return out


def layer_sweep(peaks: dict) -> dict:
    """BASELINE configs[1] at M in {1, 4, 16} (our W4A16, our FP8, cuBLAS fp16) and configs[2]
    (RMSNorm with and without residual, SwiGLU, M in {1, 16, 2048}), three sweeps with the median,
    min/max spread and the >10% flag (kernels/bench/sweep.py). A failure is recorded in the line
    rather than ending the benchmark."""
    from kernels import _lib
    from kernels.bench import sweep

    t0 = time.perf_counter()
    try:
        rows = sweep.run(sweep.KERNELS, sweeps=3)
        agg = sweep.aggregate(rows, peaks["hbm_gbs"], peaks["bf16_tflops"])
        out = {"method": "harness.time_rotating per case (CUDA graph, all inputs rotated >= 4x L2, median of 7); "
                         "median of 3 sweeps; pct_peak of MEASURED_PEAKS hbm_gbs",
               "flagged_spreads": sum(1 for r in agg if r.get("flag_spread")), "cases": sweep.compact(agg)}
    except Exception as e:  # recorded, not hidden
        out = {"error": f"{type(e).__name__}: {e}"[:300]}
    out["seconds"] = round(time.perf_counter() - t0, 1)
    try:
        out["device_error"] = _lib.device_error()
    except Exception as e:
        out["device_error"] = f"{type(e).__name__}: {e}"[:200]
    return out


# ------------------------------------------------------------------------------ 7B tensor parallel
TP_PROMPT = 1024


def run_tp7b(args, world, rank) -> dict:
    """Qwen2.5-7B-architecture decode (28 layers, hidden 3584, 28/4 heads, MLP
    18944, vocab 152064, untied lm_head), random-init weights, all linears W4A16 g128 including
    lm_head, tensor-parallel over the N ranks (column-sharded qkv/gate_up/lm_head, row-sharded
    o_proj/down), synthetic 1024-token prompts, greedy decode under CUDA graphs. Each batch size is
    timed with the fused GEMV+allreduce kernel and with the plain GEMV followed by an NCCL allreduce.
    Strong scaling: the model is the same at every N."""
    from kernels import _lib, config
    from kernels.e2e.model import QwenRunner, make_backend, random_qwen2
    from kernels.e2e.run import GraphDecoder
    from kernels.tp import TensorParallel

    t0 = time.perf_counter()
    model = random_qwen2(config.QWEN7, dtype=torch.float16, device="cuda", seed=0)
    tp = TensorParallel(mode="fused")
    base = QwenRunner(model, make_backend("ours_lm"), max_len=MAX_LEN, batch=1, tp=tp)
    del model
    torch.cuda.empty_cache()
    setup_s = time.perf_counter() - t0
    res = {"workload": "BASELINE configs[4]: Qwen2.5-7B-architecture decode, random-init weights, W4A16 g128 "
                       "linears incl. lm_head, tensor parallel (column: qkv, gate_up, lm_head; row: o_proj, down), "
                       f"uniform random {TP_PROMPT}-token prompts, greedy decode under CUDA graphs",
           "tp": world, "scaling": "strong", "unit": "tok/s", "steps": args.steps, "warmup": max(args.warmup, 3),
           "plan": {"q_heads": base.n_heads, "kv_heads": base.n_kv, "mlp_cols": base.plan.mlp[1] - base.plan.mlp[0],
                    "vocab_rows": base.plan.vocab[1] - base.plan.vocab[0]},
           "setup_s": round(setup_s, 1), "batches": {}}
    n_layers = len(base.layers)
    for B in [int(b) for b in args.tp_batches.split(",") if b]:
        runner = base if B == 1 else base.with_batch(B)
        ids = torch.randint(0, config.QWEN7["vocab_size"], (B, TP_PROMPT),
                            generator=torch.Generator().manual_seed(3)).cuda()
        row = {}
        for mode in ("fused", "nccl"):
            tp.mode = mode
            dec = GraphDecoder(runner)
            dec.capture(ids)
            sec = max_over_ranks(time_decode(dec, ids, args.steps, max(args.warmup, 3), world), world)
            row[mode] = {"tok_s": round(B * args.steps / sec, 2), "ms_per_step": round(sec / args.steps * 1e3, 4),
                         "us_per_layer": round(sec / args.steps / n_layers * 1e6, 2)}
            del dec
        tp.mode = "fused"
        row["fused_vs_nccl"] = round(row["fused"]["tok_s"] / row["nccl"]["tok_s"], 3)
        res["batches"][str(B)] = row
        del runner
        torch.cuda.empty_cache()
    res["device_error"] = _lib.device_error()
    tp.close()
    del base
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------------------ CPU baseline
def cpu_decode_rate(model, steps: int, threads: int | None = None) -> dict:
    """The reference's CPU path on the same model: OracleRunner (dequantize-then-fp32-matmul
    linears), KV cache filled to the prompt length, `steps` timed decode tokens after one untimed."""
    from kernels import config
    from oracle.runner import OracleRunner

    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    weights = oracle_weights(model)
    cfg = config.QWEN15
    r = OracleRunner(weights, cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"],
                     cfg["rms_norm_eps"], cfg["rope_theta"], max_len=PROMPT + steps + 2)
    g = torch.Generator().manual_seed(2)
    r.k[:, :, :PROMPT] = torch.randn(r.k[:, :, :PROMPT].shape, generator=g)
    r.v[:, :, :PROMPT] = torch.randn(r.v[:, :, :PROMPT].shape, generator=g)
    tok = 1
    r.step(tok, PROMPT)
    t0 = time.perf_counter()
    for i in range(steps):
        tok = int(r.step(tok, PROMPT + 1 + i).argmax())
    sec = time.perf_counter() - t0
    return {"value": round(steps / sec, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{steps} decode tokens of the same model at cache length {PROMPT} on {threads} host threads "
                      f"(oracle/runner.py, fp32 dequantize-then-matmul linears), after 1 untimed token"}


def cpu_gemv_baseline(N: int = 17920, K: int = 1536, calls: int = 5) -> dict:
    """the reference's CPU W4A16 path (unpack, dequantize in fp16, fp32 matmul;
    kernels/quant.py:31-35, kernels/reference.py:27-45) at the Qwen2.5-1.5B gate_up shape, M = 1,
    x ~ N(0,1) and W ~ N(0,0.02) RTN int4 g128 from seed 0, with torch on all host cores
    (oracle/torch_ref.py, pinned bit for bit to the reference's dequantized weights). Quantization is
    excluded; median of `calls` after one warm-up call."""
    import oracle
    from kernels.quant import weight_bytes
    from oracle import torch_ref

    threads = os.cpu_count()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, K, generator=g).half()
    w = (torch.randn(N, K, generator=g) * 0.02).half()
    qw, s, z = (torch.from_numpy(a) for a in oracle.quantize_rtn(w.numpy(), 128))
    torch_ref.w4a16_ref(x, qw, s, z, 128)
    times = []
    for _ in range(calls):
        t0 = time.perf_counter()
        y = torch_ref.w4a16_ref(x, qw, s, z, 128)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    byts = weight_bytes(N, K) + 2 * K + 2 * N
    assert y.shape == (1, N) and bool(torch.isfinite(y).all())
    return {"value": round(sec * 1e3, 3), "unit": "ms", "gbs": round(byts / sec / 1e9, 3), "cores": threads,
            "kind": "port", "shape": {"M": 1, "N": N, "K": K},
            "sample": f"{calls} calls after 1 warm-up of the reference's w4a16_ref steps on torch CPU "
                      f"({threads} threads)"}


def oracle_weights(model) -> dict:
    """Packed int4 weights for the CPU oracle, quantized by the oracle's own torch restatement of the
    reference's RTN quantizer (oracle/torch_ref.py, kernels/quant.py:38-49) on the tensors' device,
    then moved to the host: the reference arm never loads libdecodek."""
    from oracle import torch_ref

    def q(*mods):
        w = torch.cat([mm.weight.data for mm in mods], 0)
        qw, s, z = torch_ref.quantize_rtn(w, 128)
        return (qw.cpu().numpy(), s.cpu().numpy(), z.cpu().numpy())

    def npy(t):
        return t.detach().float().cpu().numpy()

    m = model.model
    layers = []
    for layer in m.layers:
        a, mlp = layer.self_attn, layer.mlp
        layers.append({"ln1": npy(layer.input_layernorm.weight), "ln2": npy(layer.post_attention_layernorm.weight),
                       "qkv": q(a.q_proj, a.k_proj, a.v_proj),
                       "qkv_bias": torch.cat([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias]).detach().float().cpu().numpy(),
                       "o": q(a.o_proj), "gate_up": q(mlp.gate_proj, mlp.up_proj), "down": q(mlp.down_proj)})
    return {"embed": npy(m.embed_tokens.weight), "final_norm": npy(m.norm.weight), "layers": layers, "lm_head": None}


# ------------------------------------------------------------------------------ arms
def run_reference(args, world, rank):
    """Reference arm: the reference's CPU path (oracle restatement) on the host cores, rank 0 only."""
    if rank != 0:
        return None
    steps = max(1, min(args.steps, 16))
    model = build_model(args.batch) if torch.cuda.is_available() else None
    if model is None:
        return {"impl": "reference", "unavailable": "needs a GPU to generate the benchmark model's weights"}
    base = cpu_decode_rate(model, steps)
    v = base["value"]
    try:
        gemv = cpu_gemv_baseline()
    except Exception as e:  # informational beside the arm's own number
        gemv = {"error": f"{type(e).__name__}: {e}"[:200]}
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "cpu_gemv_baseline": gemv,
            "steps": steps, "warmup": 1, "ms_per_step": round(1e3 / v, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, world),
            "cpu_baseline": {**base, "value": v},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def workload_config(args, world) -> dict:
    return {"workload": "BASELINE configs[3]: Qwen2.5-1.5B-architecture decode (28 layers, hidden 1536, 12/2 heads, "
                        "MLP 8960, vocab 151936, tied fp16 lm_head), random-init weights, W4A16 g128 linears, "
                        f"uniform random {PROMPT}-token prompt, greedy decode under CUDA graphs",
            "backend": args.backend, "l2_prefetch": args.l2_prefetch, "global_batch": args.batch * world, "seq_len": PROMPT, "max_len": MAX_LEN,
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "l2": "inputs larger than L2: each step reads ~1.2 GB of weights"}


def run_ours(args, world, rank, local):
    from kernels import _lib, config
    from kernels.e2e.model import QwenRunner, make_backend
    from kernels.e2e.run import GraphDecoder

    peaks = config.peaks()
    model = build_model(args.batch)
    ids = prompt_ids(model.config.vocab_size, args.batch)
    warmup = max(args.warmup, 3)
    assert PROMPT + warmup + args.steps + 8 < MAX_LEN, "steps + warmup exceed the cache"
    runner = QwenRunner(model, make_backend(args.backend), max_len=MAX_LEN, batch=args.batch,
                        l2_prefetch=args.l2_prefetch, fused_step=args.fused_step)
    dec = GraphDecoder(runner)
    dec.capture(ids)
    fused = runner.step_kernel() is not None
    runner_head = not fused and runner._kernel_head()
    with ClockSampler(local) as clocks:
        sec = time_decode(dec, ids, args.steps, warmup, world)
    sec = max_over_ranks(sec, world)
    value = world * args.batch * args.steps / sec

    # e2e: the public per-token API with host buffers (pinned H2D of the token, D2H of the next)
    dec.prefill(ids)
    t = dec.tok.cpu()
    for _ in range(3):
        t = dec.step_host(t).clone()
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        t = dec.step_host(t).clone()
    e2e_sec = max_over_ranks(time.perf_counter() - t0, world)
    e2e_value = world * args.batch * args.steps / e2e_sec

    extras = {}
    if fused:
        roof = step_roofline(runner, sec / args.steps, PROMPT + warmup, args.steps, peaks["hbm_gbs"])
    else:
        roof = gemv_roofline(runner, peaks["hbm_gbs"])
    extras["roofline"] = {**roof, "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs, copy bandwidth)"}
    if not args.no_extras:
        if fused:  # the per-op path's dominant kernel, for comparison with earlier measurements
            extras["gemv_chain"] = gemv_roofline(runner, peaks["hbm_gbs"])
        if rank == 0:
            extras["gemv_sweep"] = gemv_sweep(peaks["hbm_gbs"])
        # fp16 cuBLAS baseline runner (the reference's fp16 backend) on the same model
        base_runner = QwenRunner(model, make_backend("fp16"), max_len=MAX_LEN, batch=args.batch)
        bdec = GraphDecoder(base_runner)
        bdec.capture(ids)
        bsec = max_over_ranks(time_decode(bdec, ids, args.steps, 3, world), world)
        fp16_value = world * args.batch * args.steps / bsec
        extras["fp16_baseline"] = {"tok_s": round(fp16_value, 1), "speedup": round(value / fp16_value, 3),
                                   "what": "reference fp16 backend (cuBLAS F.linear, torch RMSNorm/SiLU, SDPA over "
                                           "max_len) on the same model and graph decoder"}
        del bdec, base_runner
        torch.cuda.empty_cache()
        if world == 1 and rank == 0:
            extras["parity"] = parity_on_benchmark_model(model, ids)
            variants = []
            for kw in ({"backend": "ours", "batch": 1, "fused": True},
                       {"backend": "ours", "batch": 1, "l2_prefetch": True},
                       {"backend": "ours", "batch": 4},
                       {"backend": "ours", "batch": 4, "fused": True},
                       {"backend": "ours", "batch": 16},
                       {"backend": "ours", "batch": 32},
                       {"backend": "ours_fp8", "batch": 1},
                       {"backend": "ours_fp8", "batch": 16},
                       {"backend": "ours_lm", "batch": 1}):
                try:
                    variants.append(decode_variant(model, steps=args.steps, warmup=warmup, **kw))
                except Exception as e:  # recorded, not hidden
                    variants.append({**kw, "error": f"{type(e).__name__}: {e}"[:200]})
            extras["variants"] = variants
            extras["cpu_baseline"] = cpu_decode_rate(model, steps=4)
            try:
                extras["cpu_gemv_baseline"] = cpu_gemv_baseline()
            except Exception as e:  # informational: never costs the benchmark line
                extras["cpu_gemv_baseline"] = {"error": f"{type(e).__name__}: {e}"[:200]}
    assert _lib.device_error() == 0, "a kernel recorded a device-side error"
    if args.tp7b == "on" or (args.tp7b == "auto" and not args.no_extras):
        del dec, runner
        torch.cuda.empty_cache()
        extras["tp7b"] = run_tp7b(args, world, rank)
    if not args.no_extras and world == 1 and rank == 0:
        torch.cuda.empty_cache()
        extras["layer_sweep"] = layer_sweep(peaks)
    # our kernels per token: the fused step is one launch; the per-op path runs the embedding kernel,
    # per layer norm+qkv, attention, o_proj, norm+gate_up+SwiGLU, down (FP8: separate norm and SwiGLU
    # kernels, 8 per layer), then the lm_head + greedy-pick kernel (a quantized lm_head instead: the
    # final norm and its GEMV, with torch's embedding and argmax)
    if fused:
        per_step_launches = 1
    else:
        per_layer = 8 if args.backend.startswith("ours_fp8") else 5
        per_step_launches = per_layer * 28 + (2 if runner_head else 2 if args.backend.endswith("_lm") else 1)
    if rank != 0:
        return None
    metric = METRIC if args.batch == 1 else METRIC.replace("batch 1", f"batch {args.batch}")
    return {"metric": metric, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": warmup, "ms_per_step": round(sec / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "w4a16 (fp16 activations, int4 weights, fp32 accumulation)",
            "data": "synthetic (random-init weights, uniform random prompt ids)",
            "config": {**workload_config(args, world), "path": "fused decode step" if fused else "per-op kernels"},
            **extras,
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 8 * args.batch,
                    "d2h_bytes_per_step": 8 * args.batch,
                    "what": "GraphDecoder.step_host: pinned-host token -> device, graph replay, next token -> host, "
                            "host wait, every step"},
            "gpu_launches": per_step_launches * args.steps,
            "clocks": clocks.summary(), "env": env_info()}


def main():
    args = parse()
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            out = run_reference(args, world, rank)
        else:
            out = run_ours(args, world, rank, local)
        if out is not None:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
