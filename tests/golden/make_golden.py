"""Generate the golden input/output vectors that pin the oracle to the reference.

Run once, in a container that has the reference checkout:

    python tests/golden/make_golden.py --reference <path to llm-decode-kernels checkout>

It imports the reference's own modules (`kernels/quant.py`, `kernels/reference.py`,
`kernels/fp8.py`, `kernels/e2e/model.py`) from that checkout, feeds them seeded inputs and writes
the inputs and outputs to `tests/golden/*.npz`. The GPU box never has the reference, so the tests
only read these files. Every case is small (a few KB) on purpose.

Cases follow the reference's own tests:
- pack/unpack round trip and the all-15 -> int32 -1 known answer (`tests/test_quant.py:8-18`);
- `quantize_rtn` on the shapes of `tests/test_quant.py:21-31` plus hand-made groups that hit the
  edge cases of the format (constant group -> scale clamp, exact .5 ties -> half-to-even, an
  all-positive and an all-negative group -> zero clamped to 0 / 15);
- `dequantize_ref` / `w4a16_ref` on the shapes of `tests/test_w4a16.py:33-79` (with bias);
- `rmsnorm_ref` and `swiglu_ref` on the shapes of `tests/test_rmsnorm.py:14` and
  `tests/test_swiglu.py:11`;
- `quantize_fp8` / `dequantize_fp8` (`tests/test_fp8.py:26-34`) plus saturating and tiny values;
- the Qwen runner on the tiny random Qwen2 of `tests/test_runner.py:15-23`, fp16 and w4_ref
  backends (logits of a 5-token forward and 8 greedy incremental steps).
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _np(t):
    import torch

    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).cpu().numpy()
    return t.detach().cpu().numpy()


def quant_cases(out: dict):
    import torch
    from kernels.quant import pack_int4, quantize_rtn, unpack_int4, weight_bytes

    torch.manual_seed(0)
    q = torch.randint(0, 16, (64, 24), dtype=torch.int32)
    out["pack_q"] = _np(q)
    out["pack_packed"] = _np(pack_int4(q))
    out["pack_unpacked"] = _np(unpack_int4(pack_int4(q)))
    q15 = torch.full((16, 3), 15, dtype=torch.int32)
    out["pack15_packed"] = _np(pack_int4(q15))

    for i, (N, K) in enumerate([(32, 128), (40, 384), (64, 256), (48, 512), (24, 1024)]):
        torch.manual_seed(100 + i)
        w = (torch.randn(N, K) * 0.02).half()
        qw, s, z = quantize_rtn(w, 128)
        out[f"rtn{i}_w"] = _np(w)
        out[f"rtn{i}_qweight"] = _np(qw)
        out[f"rtn{i}_scales"] = _np(s)
        out[f"rtn{i}_zeros"] = _np(z)

    # Hand-made edge groups: K = 128 (one group), one column per case.
    cols = []
    cols.append(torch.full((128,), 0.25))                          # constant: scale clamps to 1e-6
    cols.append(torch.arange(128) % 16 * 1.0)                      # min 0, max 15: scale exactly 1
    ties = torch.tensor([0.5, 1.5, 2.5, 3.5, 14.5, 13.5, 0.0, 15.0] * 16)
    cols.append(ties)                                              # w/scale + zero hits .5 ties
    cols.append(torch.linspace(0.01, 0.05, 128))                   # all positive: zero -> 0
    cols.append(torch.linspace(-0.05, -0.01, 128))                 # all negative: zero -> 15
    cols.append(torch.zeros(128))                                  # all zero
    cols.append(torch.linspace(-60000.0, 60000.0, 128))            # large fp16 magnitudes
    cols.append(torch.cat([torch.full((64,), -1e-4), torch.full((64,), 3e-5)]))  # tiny, near clamp
    w = torch.stack(cols, 0).half()                                # [N=8, K=128]
    qw, s, z = quantize_rtn(w, 128)
    out["rtnedge_w"] = _np(w)
    out["rtnedge_qweight"] = _np(qw)
    out["rtnedge_scales"] = _np(s)
    out["rtnedge_zeros"] = _np(z)

    out["weight_bytes"] = np.array(
        [weight_bytes(n, k) for n, k in [(1536, 1536), (2048, 1536), (17920, 1536),
                                         (1536, 8960), (151936, 1536)]], dtype=np.int64)


def matmul_cases(out: dict):
    import torch
    from kernels.quant import quantize_rtn
    from kernels.reference import dequantize_ref, w4a16_ref

    cases = [(1, 64, 256, False), (3, 40, 128, False), (17, 96, 384, False), (2, 48, 512, True),
             (1, 132, 256, True), (5, 1000, 256, True), (16, 64, 128, False)]
    out["w4_cases"] = np.array([c[:3] + (int(c[3]),) for c in cases], dtype=np.int64)
    for i, (M, N, K, bias) in enumerate(cases):
        torch.manual_seed(200 + i)
        w = (torch.randn(N, K) * 0.02).half()
        qw, s, z = quantize_rtn(w, 128)
        x = torch.randn(M, K, dtype=torch.float16)
        b = (torch.randn(N) * 0.1).half() if bias else None
        out[f"w4_{i}_x"] = _np(x)
        out[f"w4_{i}_qweight"] = _np(qw)
        out[f"w4_{i}_scales"] = _np(s)
        out[f"w4_{i}_zeros"] = _np(z)
        if bias:
            out[f"w4_{i}_bias"] = _np(b)
        if N * K <= 64 * 384:
            out[f"w4_{i}_deq"] = _np(dequantize_ref(qw, s, z, 128))
        out[f"w4_{i}_ref"] = _np(w4a16_ref(x, qw, s, z, 128, b))


def norm_act_cases(out: dict):
    import torch
    from kernels.reference import rmsnorm_ref, swiglu_ref

    for i, (M, N) in enumerate([(1, 128), (3, 1000), (5, 1536), (2, 4104)]):
        torch.manual_seed(300 + i)
        x = torch.randn(M, N, dtype=torch.float16)
        r = torch.randn(M, N, dtype=torch.float16)
        w = (1 + 0.1 * torch.randn(N)).half()
        out[f"rms{i}_x"], out[f"rms{i}_r"], out[f"rms{i}_w"] = _np(x), _np(r), _np(w)
        out[f"rms{i}_out"] = _np(rmsnorm_ref(x, w, 1e-6))
        o, res = rmsnorm_ref(x, w, 1e-6, residual=r)
        out[f"rms{i}_out_res"], out[f"rms{i}_res"] = _np(o), _np(res)

    for i, (M, I) in enumerate([(1, 64), (3, 1000), (4, 2048), (2, 4097)]):
        torch.manual_seed(400 + i)
        g = torch.randn(M, I, dtype=torch.float16) * 3
        u = torch.randn(M, I, dtype=torch.float16)
        out[f"swi{i}_g"], out[f"swi{i}_u"] = _np(g), _np(u)
        out[f"swi{i}_out"] = _np(swiglu_ref(g, u))
    # large |gate| values: silu saturates to g (positive) or -0 (negative)
    g = torch.tensor([[-65504.0, -20.0, -10.0, -1.0, -0.0, 0.0, 1e-3, 1.0, 10.0, 20.0, 60000.0,
                       -3.0, 3.0, 0.5, -0.5, 7.0]], dtype=torch.float16)
    u = torch.full_like(g, 1.5)
    out["swiedge_g"], out["swiedge_u"], out["swiedge_out"] = _np(g), _np(u), _np(swiglu_ref(g, u))


def fp8_cases(out: dict):
    import torch
    from kernels.fp8 import dequantize_fp8, quantize_fp8

    for i, (N, K) in enumerate([(64, 256), (48, 96), (40, 128)]):
        torch.manual_seed(500 + i)
        w = (torch.randn(N, K) * 0.02).half()
        wq, s = quantize_fp8(w)
        out[f"fp8{i}_w"], out[f"fp8{i}_wq"], out[f"fp8{i}_scale"] = _np(w), _np(wq), _np(s)
        out[f"fp8{i}_deq"] = _np(dequantize_fp8(wq, s))
    cols = [torch.zeros(32), torch.full((32,), 1e-7), torch.linspace(-65504, 65504, 32),
            torch.linspace(-1, 1, 32), torch.tensor([448.0, -448.0, 1e-3] + [0.0] * 29)]
    w = torch.stack(cols, 0).half()
    wq, s = quantize_fp8(w)
    out["fp8edge_w"], out["fp8edge_wq"], out["fp8edge_scale"] = _np(w), _np(wq), _np(s)
    out["fp8edge_deq"] = _np(dequantize_fp8(wq, s))
    torch.manual_seed(510)
    x = torch.randn(3, 256, dtype=torch.float16)
    w = (torch.randn(40, 256) * 0.02).half()
    wq, s = quantize_fp8(w)
    b = (torch.randn(40) * 0.1).half()
    out["w8_x"], out["w8_wq"], out["w8_scale"], out["w8_bias"] = _np(x), _np(wq), _np(s), _np(b)
    out["w8_ref"] = _np(x.float() @ dequantize_fp8(wq, s).float().t() + b.float())


def _tiny_model(dtype):
    import torch
    import transformers

    cfg = transformers.Qwen2Config(
        vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
        tie_word_embeddings=True, rms_norm_eps=1e-6,
    )
    torch.manual_seed(0)
    return transformers.Qwen2ForCausalLM(cfg).to(dtype=dtype).eval()


def weights_digest(model) -> str:
    """sha256 over the model's state dict in name order (detects a change of HF init)."""
    h = hashlib.sha256()
    for name, t in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(t.detach().float().cpu().numpy().tobytes())
    return h.hexdigest()


def runner_cases(out: dict):
    import torch
    from kernels.e2e.model import QwenRunner, make_backend

    m32 = _tiny_model(torch.float32)
    out["runner_digest32"] = np.array(weights_digest(m32))
    torch.manual_seed(600)
    ids = torch.randint(0, 512, (1, 12))
    out["runner_ids"] = _np(ids)
    r = QwenRunner(m32, make_backend("fp16"), max_len=64)
    out["runner_fp32_logits"] = _np(r.forward(ids, torch.arange(12), all_logits=True))

    m16 = _tiny_model(torch.float16)
    out["runner_digest16"] = np.array(weights_digest(m16))
    ids5 = ids[:, :5]
    for name in ("fp16", "w4_ref", "w4_ref_lm"):
        r = QwenRunner(m16, make_backend(name), max_len=32)
        out[f"runner_{name}_logits"] = _np(r.forward(ids5, torch.arange(5), all_logits=True))
    # greedy incremental decode with w4_ref (the quantized runner's numerics, on CPU)
    r = QwenRunner(m16, make_backend("w4_ref"), max_len=32)
    logits = r.forward(ids5, torch.arange(5))
    toks = [int(logits[0, -1].argmax())]
    for t in range(5, 12):
        logits = r.forward(torch.tensor([[toks[-1]]]), torch.tensor([t]))
        toks.append(int(logits[0, -1].argmax()))
    out["runner_w4_ref_greedy"] = np.array(toks, dtype=np.int64)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    import torch

    torch.set_num_threads(4)
    for name, fn in [("quant", quant_cases), ("matmul", matmul_cases),
                     ("norm_act", norm_act_cases), ("fp8", fp8_cases), ("runner", runner_cases)]:
        out: dict = {}
        fn(out)
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **out)
        print(f"wrote {path.name}: {len(out)} arrays, {path.stat().st_size} bytes")


if __name__ == "__main__":
    main()
