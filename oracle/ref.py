"""Float references of the decode hot path, restated in numpy. TEST INFRASTRUCTURE ONLY.

Each function restates the reference's PyTorch code (file:line) with the same rounding steps:
numpy float16 arithmetic rounds every op to fp16 (computed through fp32, which is exact enough
that the double rounding is innocuous), exactly like torch's fp16 CPU ops.
"""

from __future__ import annotations

import numpy as np

from oracle import dequantize_fp8, dequantize_int4


def w4a16_ref(x, qweight, scales, zeros, group_size=128, bias=None) -> np.ndarray:
    """fp32 [M, N] = fp32(x) @ fp32(dequant(W)).T (+ fp32(bias)) (kernels/reference.py:39-45)."""
    w = dequantize_int4(qweight, scales, zeros, group_size).astype(np.float32)
    out = np.asarray(x, dtype=np.float16).astype(np.float32) @ w.T
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float16).astype(np.float32)
    return out


def w8a16_ref(x, wq, scale, bias=None) -> np.ndarray:
    """fp32 [M, N] = fp32(x) @ fp32(dequantize_fp8(wq, s)).T (+ bias) (tests/test_fp8.py:18-20,
    dequantization per kernels/fp8.py:33-35)."""
    w = dequantize_fp8(wq, scale).astype(np.float32)
    out = np.asarray(x, dtype=np.float16).astype(np.float32) @ w.T
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float16).astype(np.float32)
    return out


def rmsnorm_ref(x, weight, eps=1e-6, residual=None):
    """Qwen2RMSNorm with the optional fused residual add (kernels/reference.py:9-19).

    x = x + residual in fp16; var = mean(x^2) in fp32; out = w * fp16(x * rsqrt(var + eps)),
    the last product in fp16. Returns `out` or `(out, x + residual)`."""
    x = np.asarray(x, dtype=np.float16)
    if residual is not None:
        x = x + np.asarray(residual, dtype=np.float16)
    h = x.astype(np.float32)
    var = (h * h).mean(-1, keepdims=True, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    out = np.asarray(weight, dtype=np.float16) * (h * inv).astype(np.float16)
    return out if residual is None else (out, x)


def swiglu_ref(gate, up) -> np.ndarray:
    """fp16(silu(fp32(gate))) * up in fp16, like F.silu(gate) * up (kernels/reference.py:22-24)."""
    g = np.asarray(gate, dtype=np.float16).astype(np.float32)
    with np.errstate(over="ignore"):
        act = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float16)
    return act * np.asarray(up, dtype=np.float16)
