"""Fused RMSNorm (+ residual add) (reference kernels/rmsnorm.py).

One CTA normalizes one row; with a residual the kernel also writes `x + residual` (fp16 add), which
the next decoder block needs as its residual stream. Every element is read once and written once.
"""

from __future__ import annotations

import torch

from kernels import _lib


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, residual=None):
    """RMSNorm over the last dim. Returns `out`, or `(out, x + residual)` with a residual
    (reference kernels/rmsnorm.py:44-68)."""
    shape = x.shape
    N = shape[-1]
    x2 = x.reshape(-1, N)
    _lib.reference_assert(x2.stride(-1) == 1 and weight.is_contiguous())
    _lib.require_extent(weight.numel() == N, f"rmsnorm: weight must have {N} elements")
    _lib.require_extent(residual is None or residual.shape == shape, "rmsnorm: residual must have x's shape")
    _lib.require_cuda("rmsnorm", x, weight, residual)
    _lib.require_dtype("rmsnorm", torch.float16, x, weight, residual)
    out = torch.empty_like(x2)
    if residual is not None:
        r2 = residual.reshape(-1, N)
        if r2.stride(-1) != 1:
            r2 = r2.contiguous()
        res_out = torch.empty_like(x2)
    else:
        r2, res_out = None, None
    _lib.call("dk_rmsnorm", _lib.ptr(x2), x2.stride(0), _lib.ptr(r2), r2.stride(0) if r2 is not None else 0,
              _lib.ptr(weight), _lib.ptr(out), out.stride(0), _lib.ptr(res_out),
              res_out.stride(0) if res_out is not None else 0, x2.shape[0], N, float(eps),
              _lib.stream_of(x))
    if residual is None:
        return out.view(shape)
    return out.view(shape), res_out.view(shape)


def rmsnorm_bytes(M: int, N: int, residual: bool, elem: int = 2) -> int:
    """Minimum DRAM traffic: read x (+ residual) and weight, write out (+ new residual)
    (reference kernels/rmsnorm.py:71-74)."""
    tensors = 4 if residual else 2
    return tensors * M * N * elem + N * elem
