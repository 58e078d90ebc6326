"""The reference's CPU W4A16 path, restated with torch CPU ops (multi-threaded), for timing it.
TEST INFRASTRUCTURE AND CPU BASELINE ONLY (never the product path).

Same steps as kernels/quant.py:31-35 (unpack: arithmetic shift by 4i, mask 0xF) and
kernels/reference.py:27-45 (dequantize: `(q.to(fp16) - z) * s` in fp16 with scales and zeros
repeated over each group, transposed to [N, K]; matmul: `x.float() @ W.float().t()`). The results
are pinned bit for bit against the C restatement (`oracle.dequantize_int4`) by tests/test_oracle.py.
"""

from __future__ import annotations

import torch


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """int32 [K/8, N] -> int32 [K, N]: nibble i of each word is K index 8r + i."""
    shifts = torch.arange(0, 32, 4, dtype=torch.int32).view(1, 8, 1)
    return ((packed.unsqueeze(1) >> shifts) & 0xF).reshape(-1, packed.shape[1])


def dequantize(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """-> fp16 [N, K]."""
    q = unpack_int4(qweight)
    s = scales.repeat_interleave(group_size, dim=0)
    z = zeros.repeat_interleave(group_size, dim=0)
    return ((q.to(torch.float16) - z) * s).t()


def w4a16_ref(x: torch.Tensor, qweight, scales, zeros, group_size: int = 128, bias=None) -> torch.Tensor:
    """fp32 [M, N] = x.float() @ dequant(W).float().t() (+ bias)."""
    out = x.float() @ dequantize(qweight, scales, zeros, group_size).float().t()
    if bias is not None:
        out = out + bias.float()
    return out
