"""Host logic of the layer sweep (kernels/bench/sweep.py): the case inventory, the algorithmic bytes
(the reference's formulas, kernels/bench/sweep.py:167-169 and kernels/quant.py:52-54), and the
median / spread aggregation over sweeps (reference kernels/bench/sweep.py:206-233). CPU only."""

import pytest

from kernels.bench import sweep


def test_case_inventory():
    specs = sweep.case_specs()
    kinds = [s["kernel"] for s in specs]
    assert kinds.count("copy") == 1
    assert kinds.count("rmsnorm") == 6  # M in {1, 16, 2048} x residual or not
    assert kinds.count("swiglu") == 3
    assert kinds.count("w4a16") == 5 * 3 * 3  # 5 Qwen2.5-1.5B shapes x M in {1, 4, 16} x 3 impls
    w4 = {(s["shape"]["layer"], s["shape"]["M"], s["impl"]) for s in specs if s["kernel"] == "w4a16"}
    assert ("lm_head", 16, "fp8") in w4 and ("down", 4, "fp16") in w4
    assert len(sweep.case_specs(("w4a16",), quick=True)) == 2 * 3 * 3
    with pytest.raises(ValueError):
        sweep.case_specs(("gemm",))


def test_algorithmic_bytes():
    def spec(kernel, impl, **shape):
        return {"kernel": kernel, "impl": impl, "shape": shape}

    # W4A16 at M = 1: x + y + packed weights, scales and zeros (qkv, lm_head of Qwen2.5-1.5B)
    assert sweep.bytes_and_flops(spec("w4a16", "ours", layer="qkv", M=1, N=2048, K=1536)) == (1678336, 2 * 2048 * 1536)
    assert sweep.bytes_and_flops(spec("w4a16", "ours", layer="lm_head", M=1, N=151936, K=1536))[0] == 124286720
    # fp16 reads 2 bytes per weight, FP8 one plus a scale per column
    assert sweep.bytes_and_flops(spec("w4a16", "fp16", layer="o", M=1, N=1536, K=1536))[0] == 3072 + 3072 + 1536 * 1536 * 2
    assert sweep.bytes_and_flops(spec("w4a16", "fp8", layer="o", M=1, N=1536, K=1536))[0] == 3072 + 3072 + 1536 * 1536 + 3072
    assert sweep.bytes_and_flops(spec("rmsnorm", "ours", M=16, N=1536, residual=True)) == (4 * 16 * 1536 * 2 + 2 * 1536, 0)
    assert sweep.bytes_and_flops(spec("swiglu", "ours", M=2048, I=8960)) == (3 * 2048 * 8960 * 2, 0)
    assert sweep.bytes_and_flops(spec("copy", "torch", elems=1024)) == (4096, 0)


def test_aggregate_median_spread_and_errors():
    shape = {"layer": "qkv", "M": 1, "N": 2048, "K": 1536}
    rows = [{"kernel": "w4a16", "impl": "ours", "shape": shape, "sweep": i, "ms": ms}
            for i, ms in enumerate([0.0030, 0.0036, 0.0033])]
    rows += [{"kernel": "swiglu", "impl": "ours", "shape": {"M": 1, "I": 8960}, "sweep": i, "ms": 0.002} for i in range(3)]
    rows += [{"kernel": "swiglu", "impl": "ours", "shape": {"M": 16, "I": 8960}, "sweep": 0, "error": "RuntimeError: x"}]
    agg = sweep.aggregate(rows, peak_gbs=1000.0, peak_tflops=100.0)
    assert [r["kernel"] for r in agg] == ["w4a16", "swiglu", "swiglu"]
    a = agg[0]
    assert a["sweeps"] == 3 and a["us"] == 3.3 and a["us_min"] == 3.0 and a["us_max"] == 3.6
    assert a["spread_pct"] == pytest.approx(18.2, abs=0.05) and a["flag_spread"]
    assert a["gbs"] == pytest.approx(1678336 / 3.3e-6 / 1e9, rel=1e-3)
    assert a["pct_peak"] == pytest.approx(100 * a["gbs"] / 1000.0, abs=0.1)
    assert a["tflops"] == pytest.approx(2 * 2048 * 1536 / 3.3e-6 / 1e12, abs=0.01)
    assert not agg[1]["flag_spread"] and agg[1]["spread_pct"] == 0.0
    assert agg[2]["sweeps"] == 0 and agg[2]["error"].startswith("RuntimeError")
    c = sweep.compact(agg)
    assert set(c) == {"w4a16/ours/qkv/M1", "swiglu/M1", "swiglu/M16"}
    assert c["w4a16/ours/qkv/M1"]["us"] == 3.3 and "error" in c["swiglu/M16"]


def test_run_records_failures_and_goes_on(monkeypatch):
    """A case that raises is recorded with its error and the sweep continues (fake timer, CPU)."""
    calls = []

    def fake_time(spec, weights):
        calls.append(spec["kernel"])
        if spec["kernel"] == "swiglu" and spec["shape"]["M"] == 16:
            raise RuntimeError("no tile")
        return 0.001

    monkeypatch.setattr(sweep, "time_case", fake_time)
    rows = sweep.run(("rmsnorm", "swiglu"), sweeps=2)
    assert len(rows) == 2 * (6 + 3) and len(calls) == len(rows)
    bad = [r for r in rows if "error" in r]
    assert len(bad) == 2 and all(r["shape"]["M"] == 16 for r in bad)
    agg = sweep.aggregate(rows, 1000.0, 100.0)
    assert len(agg) == 9 and sum("error" in r for r in agg) == 1


def test_bench_line_layer_sweep(monkeypatch):
    """bench.py's layer_sweep entry: compact cases, the spread count, and a failure recorded in the
    line instead of ending the benchmark."""
    import bench
    from kernels import _lib

    monkeypatch.setattr(_lib, "device_error", lambda: 0)
    monkeypatch.setattr(sweep, "time_case", lambda spec, weights: 0.002)
    out = bench.layer_sweep({"hbm_gbs": 6000.0, "bf16_tflops": 1600.0})
    assert out["device_error"] == 0 and out["flagged_spreads"] == 0
    assert len(out["cases"]) == len(sweep.case_specs())
    assert "w4a16/fp16/lm_head/M16" in out["cases"] and "rmsnorm/M2048/residual" in out["cases"]

    def boom(*a, **k):
        raise RuntimeError("CUDA error: out of memory")

    monkeypatch.setattr(sweep, "run", boom)
    out = bench.layer_sweep({"hbm_gbs": 6000.0, "bf16_tflops": 1600.0})
    assert out["error"].startswith("RuntimeError") and "seconds" in out


def test_bench_cpu_gemv_baseline_small():
    """bench.py's configs[0] CPU baseline (the reference's w4a16_ref steps on torch CPU) on a small
    shape: a median time in ms, the bandwidth it implies and the thread count."""
    import bench

    out = bench.cpu_gemv_baseline(N=256, K=256, calls=2)
    assert out["unit"] == "ms" and out["value"] > 0 and out["cores"] >= 1 and out["kind"] == "port"
    assert out["shape"] == {"M": 1, "N": 256, "K": 256}


def test_checkpoint_resumes_without_measuring_again(monkeypatch, tmp_path):
    """Rows go to the checkpoint as they finish; a rerun reuses them and measures only what is
    missing (the reference's resumable sweeps)."""
    ck = str(tmp_path / "sweep.jsonl")
    calls = []

    def timer(spec, weights):
        calls.append(spec["kernel"])
        if len(calls) == 5:
            raise KeyboardInterrupt  # the first run is interrupted after 4 cases
        return 0.001 * len(calls)

    monkeypatch.setattr(sweep, "time_case", timer)
    with pytest.raises(KeyboardInterrupt):
        sweep.run(("rmsnorm",), sweeps=1, checkpoint=ck)
    assert len(open(ck).read().splitlines()) == 4
    calls.clear()
    monkeypatch.setattr(sweep, "time_case", lambda spec, weights: calls.append(1) or 0.5)
    rows = sweep.run(("rmsnorm",), sweeps=1, checkpoint=ck)
    assert len(rows) == 6 and len(calls) == 2  # only the two unfinished cases were measured
    assert [r["ms"] for r in rows[:4]] == [0.001, 0.002, 0.003, 0.004]
    assert len(open(ck).read().splitlines()) == 6


def test_bench_env_info():
    """The bench line's env entry (versions, host cores; GPU fields where a GPU is present) never
    raises, even without nvidia-smi."""
    import bench

    env = bench.env_info()
    assert env["torch"] and env["host_cpus"] >= 1 and "python" in env
