"""Small, self-terminating workloads for profiler captures (ncu launch lists and single-kernel reports).

    python llm-decode-kernels_b200/kernels/bench/profile_cases.py decode [ours|fp16] [steps] [l2_prefetch 0|1] [batch]
        Qwen2.5-1.5B (random init) batch-1 decode through the CUDA graph; the profiler range
        (cudaProfilerStart/Stop) covers exactly `steps` graph replays at context 512.
    python .../profile_cases.py gemv_layer
        one decoder layer's four W4A16 launches at the Qwen2.5-1.5B shapes (M=1), as the runner
        issues them (norm+qkv, o_proj, norm+gate_up+SwiGLU, down), 3 warm-up rounds + 1.
    python .../profile_cases.py gemv N K [M]
        five launches of one W4A16 GEMV of shape [M, K] x [K, N].
    python .../profile_cases.py gemm M N K
        three launches of the tcgen05 W4A16 GEMM of shape [M, K] x [K, N], then 20 timed ones.
    python .../profile_cases.py chain [n]
        the cost of a kernel boundary: n tiny launches in one CUDA graph, with and without PDL.
    python .../profile_cases.py attention [pos] [splits]
        28 decode-attention launches (one per layer, Qwen2.5-1.5B heads, position 767 by default,
        automatic split) eagerly, then as a CUDA graph replayed 21 times.
    python .../profile_cases.py config_sweep [M]
        the cost model's GEMV choice against every BLOCK_N x SPLIT_K of one decoder layer's four
        launches, and the lm_head-shaped GEMV at three widths.
    python .../profile_cases.py head [rows] [launches]
        the lm_head + greedy-pick kernel on the tied Qwen2.5-1.5B lm_head, timed (CUDA events) against
        cuBLAS F.linear + torch.argmax; the profiler range holds the kernel's timed launches.
    python .../profile_cases.py step [layers] [steps] [batch]
        the fused decode-step kernel on a Qwen2.5-1.5B-shaped model with `layers` layers (4 by
        default: ~0.6 GB of weights incl. the fp16 lm_head) at context 512: 3 warm-up steps, then
        `steps` steps (eager launches, inside the profiler range).

Every case allocates at most a few hundred MB and ends by itself.
"""

from __future__ import annotations

import os
import sys

# run as a script, this directory would come first on sys.path and its profile.py would shadow the
# standard library's `profile` (which torch imports through cProfile)
_here = os.path.dirname(os.path.abspath(__file__))
sys.path = [q for q in sys.path if os.path.abspath(q or ".") != _here]
sys.path.insert(0, os.path.abspath(os.path.join(_here, "..", "..")))

import torch  # noqa: E402

from kernels import config  # noqa: E402
from kernels.attention import decode_attention  # noqa: E402
from kernels.quant import quantize_rtn  # noqa: E402
from kernels.w4a16 import w4a16_matmul, w4a16_rmsnorm_matmul  # noqa: E402


def _q(N, K):
    return quantize_rtn((torch.randn(N, K, device="cuda") * 0.02).half(), config.GROUP_SIZE)


def decode(backend="ours", steps="2", l2_prefetch="0", batch="1"):
    from kernels.e2e.model import QwenRunner, make_backend, random_qwen2
    from kernels.e2e.run import GraphDecoder
    steps, batch = int(steps), int(batch)
    model = random_qwen2(config.QWEN15, dtype=torch.float16, device="cuda", seed=0)
    ids = torch.randint(0, config.QWEN15["vocab_size"], (batch, 512), device="cuda")
    dec = GraphDecoder(QwenRunner(model, make_backend(backend), max_len=2048, batch=batch,
                                  l2_prefetch=l2_prefetch != "0"))
    dec.capture(ids)
    dec.prefill(ids)
    for _ in range(5):
        dec.graph.replay()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(steps):
        dec.graph.replay()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(50):
        dec.graph.replay()
    e1.record()
    torch.cuda.synchronize()
    print(f"{backend} (l2_prefetch={l2_prefetch}): {e0.elapsed_time(e1) / 50:.4f} ms/step")


def gemv_layer():
    H, I, NQKV = 1536, 8960, 2048
    qkv, o, gu, dn = _q(NQKV, H), _q(H, H), _q(2 * I, H), _q(H, I)
    bias = (torch.randn(NQKV, device="cuda") * 0.1).half()
    ln = torch.ones(H, device="cuda").half()
    x, r, a = (torch.randn(1, H, device="cuda").half() for _ in range(3))
    cfg = {"STATIC_WEIGHTS": True}

    def layer():
        w4a16_rmsnorm_matmul(x, ln, 1e-6, r, *qkv, bias=bias, config=cfg)
        w4a16_matmul(a, *o, config=cfg)
        act, _ = w4a16_rmsnorm_matmul(x, ln, 1e-6, r, *gu, swiglu=True, config=cfg)
        w4a16_matmul(act, *dn, config=cfg)

    for _ in range(4):
        layer()
    torch.cuda.synchronize()
    print("gemv_layer ok")


def gemv(N, K, M="1"):
    N, K, M = int(N), int(K), int(M)
    qw, s, z = _q(N, K)
    x = torch.randn(M, K, device="cuda").half()
    for _ in range(5):
        y = w4a16_matmul(x, qw, s, z)
    torch.cuda.synchronize()
    print("gemv ok", y.float().abs().mean().item())


def gemm(M, N, K):
    M, N, K = int(M), int(N), int(K)
    qw, s, z = _q(N, K)
    x = torch.randn(M, K, device="cuda").half()
    for _ in range(3):
        w4a16_matmul(x, qw, s, z)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(20):
        w4a16_matmul(x, qw, s, z)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    print(f"gemm M={M} N={N} K={K}: {ms * 1e3:.1f} us, {2 * M * N * K / ms / 1e9:.1f} TFLOP/s")


def chain(n="200"):
    """Cost of a kernel boundary: a CUDA graph of `n` back-to-back launches of the smallest
    libdecodek kernel (SwiGLU of one 16-wide row), with programmatic dependent launch on and off."""
    from kernels import _lib
    from kernels.bench.harness import capture
    from kernels.swiglu import swiglu_fused

    n = int(n)
    x = torch.randn(1, 32, device="cuda").half()
    for pdl in (1, 0):
        _lib.set_pdl(bool(pdl))
        swiglu_fused(x)
        torch.cuda.synchronize()
        graph, _ = capture(lambda: [swiglu_fused(x) for _ in range(n)])
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(10):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        print(f"chain of {n} tiny launches, pdl={pdl}: {e0.elapsed_time(e1) / 10 / n * 1e3:.3f} us per launch")
        del graph
    _lib.set_pdl(True)


def attention(pos="767", splits="0"):
    a = config.QWEN15
    nq, nkv, hd = a["num_attention_heads"], a["num_key_value_heads"], a["head_dim"]
    layers, max_len, pos, splits = a["num_hidden_layers"], 2048, int(pos), int(splits)
    qkv = torch.randn(1, 1, (nq + 2 * nkv) * hd, device="cuda").half()
    kc = torch.randn(layers, 1, nkv, max_len, hd, device="cuda").half()
    vc = torch.randn(layers, 1, nkv, max_len, hd, device="cuda").half()
    p = torch.tensor([pos], device="cuda")
    cos = torch.randn(1, hd, device="cuda").half()
    sin = torch.randn(1, hd, device="cuda").half()

    def run():
        for i in range(layers):
            decode_attention(qkv, kc[i], vc[i], p, cos, sin, nq, nkv, splits=splits, static_cache=True)

    run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(20):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    print(f"attention: {e0.elapsed_time(e1) * 1e3 / (20 * layers):.2f} us/launch (position {pos}, splits {splits})")


def small_m():
    """us per launch of W4A16 at M = 16 and 32 on the Qwen2.5-1.5B shapes: the tcgen05 small-M kernel
    (default) against 16-row launches of the decode GEMV (DECODE_GEMV), CUDA graph of 20 launches."""
    from kernels.bench.harness import capture

    for label, N, K in config.QWEN15_SHAPES[:4]:
        qw, s, z = _q(N, K)
        for M in (16, 32):
            x = torch.randn(M, K, device="cuda").half()
            res = []
            for cfg in ({"STATIC_WEIGHTS": True}, {"STATIC_WEIGHTS": True, "DECODE_GEMV": True}):
                w4a16_matmul(x, qw, s, z, config=cfg)
                torch.cuda.synchronize()
                graph, _ = capture(lambda: [w4a16_matmul(x, qw, s, z, config=cfg) for _ in range(20)])
                graph.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                e0.record()
                for _ in range(5):
                    graph.replay()
                e1.record()
                torch.cuda.synchronize()
                res.append(e0.elapsed_time(e1) / 100 * 1e3)
                del graph
            print(f"{label} {N}x{K} M={M}: tcgen05 small-M {res[0]:.2f} us, decode GEMV {res[1]:.2f} us")


def attention_sweep():
    """Decode attention us/launch over positions x cluster splits (one process)."""
    for pos in ("511", "1023", "2047"):
        for splits in ("2", "4", "8", "16"):
            attention(pos, splits)


def config_sweep(M="1"):
    """The static cost model's choice against the BLOCK_N x SPLIT_K space: us per launch of the four
    W4A16 launches of a Qwen2.5-1.5B decoder layer as the runner issues them (norm+qkv, o_proj,
    norm+gate_up+SwiGLU, down) at M rows, for BLOCK_N in {auto, 32, 64, 128, 256} and the split-K
    factors K allows; then the lm_head-shaped GEMV at three widths (the slope is its marginal
    bandwidth). Timed like the reference's harness (CUDA graph, rotating weight copies >= 4x L2)."""
    from kernels.bench.harness import time_rotating

    M = int(M)
    H, inter = config.QWEN15["hidden_size"], config.QWEN15["intermediate_size"]
    x = torch.randn(M, H, device="cuda").half()
    res = torch.randn(M, H, device="cuda").half()
    nw = (1 + 0.05 * torch.randn(H, device="cuda")).half()
    xd = torch.randn(M, inter, device="cuda").half()

    def op(kind, cfg):
        if kind == "norm":
            return lambda xx, q, s, z: w4a16_rmsnorm_matmul(xx, nw, 1e-6, res, q, s, z, config=cfg)
        if kind == "norm_swiglu":
            return lambda xx, q, s, z: w4a16_rmsnorm_matmul(xx, nw, 1e-6, res, q, s, z, swiglu=True, config=cfg)
        return lambda xx, q, s, z: w4a16_matmul(xx, q, s, z, config=cfg)

    layer = [("norm+qkv", "norm", 2048, H, x), ("o_proj", "plain", H, H, x),
             ("norm+gate_up+swiglu", "norm_swiglu", 2 * inter, H, x), ("down", "plain", H, inter, xd)]
    for label, kind, N, K, xin in layer:
        qw, s, z = _q(N, K)
        stages = (K + 255) // 256
        # the split-K factors the kernel accepts as given (every cluster rank gets a stage)
        splits = [0] + [sp for sp in range(1, 9) if sp <= stages and (sp - 1) * -(-stages // sp) < stages]
        rows = []
        for bn in (0, 32, 64, 128, 256):
            for sp in splits:
                cfg = {"STATIC_WEIGHTS": True, "BLOCK_N": bn, "SPLIT_K": sp}
                us = time_rotating(op(kind, cfg), (xin, qw, s, z), rotate=(1, 2, 3)) * 1e3
                rows.append((us, bn, sp))
                print(f"M={M} {label} BLOCK_N={bn or 'auto'} SPLIT_K={sp or 'auto'}: {us:.2f} us", flush=True)
        auto = rows[0][0]
        best = min(rows)
        print(f"M={M} {label}: auto {auto:.2f} us, best {best[0]:.2f} us (BLOCK_N={best[1] or 'auto'}, "
              f"SPLIT_K={best[2] or 'auto'})", flush=True)
        del qw, s, z
        torch.cuda.empty_cache()
    for N in (37984, 75968, 151936):
        qw, s, z = _q(N, H)
        us = time_rotating(op("plain", {"STATIC_WEIGHTS": True}), (x[:1], qw, s, z), rotate=(1, 2, 3)) * 1e3
        print(f"lm_head-shaped GEMV N={N} K={H} M=1: {us:.2f} us", flush=True)
        del qw, s, z
        torch.cuda.empty_cache()


def step(layers="4", steps="2", batch="1"):
    from kernels.e2e.model import QwenRunner, make_backend, random_qwen2
    from kernels.e2e.run import GraphDecoder
    layers, steps, batch = int(layers), int(steps), int(batch)
    arch = dict(config.QWEN15, num_hidden_layers=layers)
    model = random_qwen2(arch, dtype=torch.float16, device="cuda", seed=0)
    ids = torch.randint(0, arch["vocab_size"], (batch, 512), device="cuda")
    runner = QwenRunner(model, make_backend("ours"), max_len=2048, batch=batch, fused_step=True)
    dec = GraphDecoder(runner)
    dec.prefill(ids)
    kernel = runner.step_kernel()
    assert kernel is not None, "fused step unavailable"
    for _ in range(3):
        kernel(dec.tok, dec.pos, dec.out)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(steps):
        kernel(dec.tok, dec.pos, dec.out)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    from kernels import _lib
    assert _lib.device_error() == 0
    print("step ok", dec.pos.item())


def head(rows="1", launches="50"):
    """The lm_head + greedy-pick kernel on the tied Qwen2.5-1.5B lm_head (151936 x 1536 fp16,
    467 MB: larger than L2 by itself): 3 warm-up launches, then `launches` timed with CUDA events
    inside the profiler range, against cuBLAS F.linear + torch.argmax on the same operands."""
    from kernels import _lib
    from kernels import head as hd
    import torch.nn.functional as F

    M, n = int(rows), int(launches)
    V, H = config.QWEN15["vocab_size"], config.QWEN15["hidden_size"]
    W = (torch.randn(V, H, device="cuda") * 0.05).half()
    x, res = torch.randn(M, H, device="cuda").half(), torch.randn(M, H, device="cuda").half()
    w = torch.ones(H, device="cuda").half()
    ws, tok = hd.workspace("cuda"), torch.empty(M, dtype=torch.int64, device="cuda")
    out = {}
    for name, fn in (("lm_head_greedy", lambda: hd.lm_head_greedy(x, res, w, 1e-6, W, tok, ws)),
                     ("cublas_linear_argmax", lambda: F.linear(x, W).argmax(-1))):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        if name == "lm_head_greedy":
            torch.cuda.profiler.start()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        if name == "lm_head_greedy":
            torch.cuda.profiler.stop()
        us = e0.elapsed_time(e1) / n * 1e3
        out[name] = f"{us:.2f} us, {V * H * 2 / us / 1e3:.0f} GB/s"
    assert _lib.device_error() == 0
    print(f"rows {M}:", out)


CASES = {"head": head, "step": step, "decode": decode, "gemv_layer": gemv_layer, "gemv": gemv, "attention": attention, "gemm": gemm, "chain": chain, "attention_sweep": attention_sweep, "small_m": small_m, "config_sweep": config_sweep}

if __name__ == "__main__":
    if len(sys.argv) < 2 or sys.argv[1] not in CASES:
        sys.exit(f"usage: profile_cases.py {{{'|'.join(CASES)}}} [args]")
    CASES[sys.argv[1]](*sys.argv[2:])
