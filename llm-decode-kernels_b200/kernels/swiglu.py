"""Fused SwiGLU activation: out = silu(gate) * up in one pass (reference kernels/swiglu.py).

Accepts two tensors or one fused [.., 2*I] tensor (gate first, then up), read in place.
"""

from __future__ import annotations

import torch

from kernels import _lib


def _launch(gate2: torch.Tensor, up2: torch.Tensor) -> torch.Tensor:
    M, I = gate2.shape
    _lib.reference_assert(gate2.stride(-1) == 1 and up2.stride(-1) == 1)
    _lib.require_cuda("swiglu", gate2, up2)
    _lib.require_dtype("swiglu", torch.float16, gate2, up2)
    out = torch.empty((M, I), dtype=gate2.dtype, device=gate2.device)
    _lib.call("dk_swiglu", _lib.ptr(gate2), gate2.stride(0), _lib.ptr(up2), up2.stride(0), _lib.ptr(out),
              out.stride(0), M, I, _lib.stream_of(gate2))
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up for two same-shape tensors (reference kernels/swiglu.py:49-53)."""
    _lib.require_extent(gate.shape == up.shape, "swiglu: gate and up must have the same shape")
    I = gate.shape[-1]
    out = _launch(gate.reshape(-1, I), up.reshape(-1, I))
    return out.view(gate.shape)


def swiglu_fused(gate_up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up where gate_up = cat([gate, up], dim=-1); halves read in place
    (reference kernels/swiglu.py:56-61)."""
    I = gate_up.shape[-1] // 2
    gu = gate_up.reshape(-1, 2 * I)
    out = _launch(gu[:, :I], gu[:, I:])
    return out.view(*gate_up.shape[:-1], I)


def swiglu_bytes(M: int, I: int, elem: int = 2) -> int:
    """Read gate and up, write out (reference kernels/swiglu.py:64-65)."""
    return 3 * M * I * elem
