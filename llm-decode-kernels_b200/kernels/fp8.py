"""FP8 (e4m3) weight-only matmul (W8A16): y = x @ (Wq * s).T (+ bias) (reference kernels/fp8.py).

Weights are float8 e4m3 with one fp16 scale per output channel, stored as [K, N] (N contiguous,
like the int4 format). The scale factors out of the K sum and multiplies the fp32 result. All
functions run libdecodek kernels; quantize_fp8 / dequantize_fp8 are bit-exact with the reference.
`config` accepts the reference's Triton dicts: SPLIT_K / BLOCK_N map to the cluster split and the
column tile, the other keys are accepted and ignored.
"""

from __future__ import annotations

import ctypes

import torch

from kernels import _lib
from kernels.w4a16 import _config

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0


def quantize_fp8(weight: torch.Tensor):
    """[N, K] fp16 -> (wq float8 [K, N], scale fp16 [N]), per-output-channel absmax scaling
    (reference kernels/fp8.py:25-30)."""
    _lib.require_cuda("quantize_fp8", weight)
    _lib.require_dtype("quantize_fp8", torch.float16, weight)
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    N, K = weight.shape
    wq = torch.empty((K, N), dtype=FP8, device=weight.device)
    s = torch.empty((N,), dtype=weight.dtype, device=weight.device)
    _lib.call("dk_quantize_fp8", _lib.ptr(weight), weight.stride(0), _lib.ptr(wq), _lib.ptr(s), N, K,
              _lib.stream_of(weight))
    return wq, s


def dequantize_fp8(wq: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """-> [N, K] in scale's dtype (reference kernels/fp8.py:33-35)."""
    _lib.require_cuda("dequantize_fp8", wq, scale)
    K, N = wq.shape
    out = torch.empty((N, K), dtype=scale.dtype, device=wq.device)
    _lib.call("dk_dequantize_fp8", _lib.ptr(wq.contiguous()), _lib.ptr(scale.contiguous()), _lib.ptr(out), N, K,
              _lib.stream_of(wq))
    return out


def fp8_bytes(N: int, K: int) -> int:
    """e4m3 weight bytes + fp16 scales (reference kernels/fp8.py:38-39)."""
    return N * K + N * 2


def w8a16_matmul(x, wq, scale, bias=None, config=None):
    """y = x @ (wq * scale).T (+ bias). x: [..., K] fp16, wq: float8 [K, N], scale: fp16 [N]
    (reference kernels/fp8.py:200-223)."""
    K = x.shape[-1]
    N = wq.shape[1]
    _lib.require_extent(wq.shape[0] == K, f"w8a16_matmul: wq must be [{K}, N]")
    _lib.require_extent(tuple(scale.shape) == (N,), f"w8a16_matmul: scale must be [{N}]")
    _lib.require_extent(bias is None or tuple(bias.shape) == (N,), f"w8a16_matmul: bias must be [{N}]")
    _lib.require_cuda("w8a16_matmul", x, wq, scale, bias)
    _lib.require_dtype("w8a16_matmul", torch.float16, x, scale, bias)
    _lib.require_dtype("w8a16_matmul", FP8, wq)
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    wq, scale = wq.contiguous(), scale.contiguous()
    if bias is not None:
        bias = bias.contiguous()
    M = x2.shape[0]
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    cfg = _config(config)
    _lib.call("dk_w8a16_matmul", _lib.ptr(x2), x2.stride(0), _lib.ptr(wq), _lib.ptr(scale), _lib.ptr(bias),
              _lib.ptr(out), out.stride(0), M, N, K, ctypes.byref(cfg), _lib.stream_of(x))
    return out.view(*x.shape[:-1], N)
