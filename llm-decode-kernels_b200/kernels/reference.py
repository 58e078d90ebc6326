"""PyTorch references used by the runner's baseline backends (reference kernels/reference.py).

`fp16` runs plain torch ops (cuBLAS F.linear, this RMSNorm, F.silu) and `w4_ref` dequantizes the
4-bit weights once and then uses cuBLAS; both are the comparison baselines of the decode benchmark,
not the product path. `dequantize_ref` runs libdecodek's dequantization kernel (same fp16 rounding
as the reference: `(q.to(fp16) - z) * s`).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from kernels import _lib


def rmsnorm_ref(x, weight, eps=1e-6, residual=None):
    """Qwen2RMSNorm, optionally preceded by the residual add (reference kernels/reference.py:9-19).
    Returns `out`, or `(out, x + residual)` when `residual` is given."""
    if residual is not None:
        x = x + residual  # fp16 add, as in the HF decoder layer
    h = x.float()
    var = h.pow(2).mean(-1, keepdim=True)
    out = weight * (h * torch.rsqrt(var + eps)).to(x.dtype)
    return out if residual is None else (out, x)


def swiglu_ref(gate, up):
    """Qwen2MLP activation: silu(gate) * up in fp16 (reference kernels/reference.py:22-24)."""
    return F.silu(gate) * up


def dequantize_ref(qweight, scales, zeros, group_size=128):
    """Unpack int4 weights to fp16 with layout [N, K] (reference kernels/reference.py:27-36)."""
    _lib.require_cuda("dequantize_ref", qweight, scales, zeros)
    K, N = qweight.shape[0] * 8, qweight.shape[1]
    out = torch.empty((N, K), dtype=scales.dtype, device=qweight.device)
    _lib.call("dk_dequantize_int4", _lib.ptr(qweight.contiguous()), _lib.ptr(scales.contiguous()),
              _lib.ptr(zeros.contiguous()), _lib.ptr(out), N, K, group_size, _lib.stream_of(qweight))
    return out


def w4a16_ref(x, qweight, scales, zeros, group_size=128, bias=None):
    """fp32 reference: x @ dequant(W).T (+ bias) (reference kernels/reference.py:39-45)."""
    w = dequantize_ref(qweight, scales, zeros, group_size)
    out = x.float() @ w.float().t()
    if bias is not None:
        out = out + bias.float()
    return out
