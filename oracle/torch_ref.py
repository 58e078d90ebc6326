"""The reference's CPU path for the hot-path ops, restated with torch CPU ops (multi-threaded): to
time the CPU baseline and to cross-check the C / numpy oracle on many inputs.
TEST INFRASTRUCTURE AND CPU BASELINE ONLY (never the product path).

Same steps as kernels/quant.py:20-49 (pack, RTN quantization, unpack: arithmetic shift by 4i, mask
0xF), kernels/fp8.py:25-30 (e4m3 quantization) and kernels/reference.py:9-45 (RMSNorm, SwiGLU;
dequantize: `(q.to(fp16) - z) * s` in fp16 with scales and zeros repeated over each group,
transposed to [N, K]; matmul: `x.float() @ W.float().t()`). tests/test_oracle.py pins these against
the golden vectors and checks them against the C / numpy oracle.
"""

from __future__ import annotations

import torch


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """[K, N] integers 0..15 -> int32 [K/8, N]: value i of 8 consecutive K rows in bits 4i..4i+3 of a
    32-bit word, read as a signed int32 (kernels/quant.py:20-28)."""
    K, N = q.shape
    rows = q.to(torch.int64).reshape(K // 8, 8, N)
    word = (rows << torch.arange(0, 32, 4, dtype=torch.int64, device=q.device).view(1, 8, 1)).sum(dim=1)
    return (word - ((word >> 31) << 32)).to(torch.int32)


def quantize_rtn(weight: torch.Tensor, group_size: int = 128):
    """fp16 [N, K] -> (qweight int32 [K/8, N], scales fp16 [K/g, N], zeros fp16 [K/g, N]): per group of
    `group_size` K values and column, fp32 min and max, scale = (max - min) / 15 clamped to >= 1e-6,
    zero = round(-min / scale) clamped to 0..15, q = round(w / scale + zero) clamped to 0..15, rounding
    half to even (kernels/quant.py:38-49)."""
    N, K = weight.shape
    w = weight.t().float().reshape(K // group_size, group_size, N)
    lo, hi = w.amin(dim=1), w.amax(dim=1)
    scale = ((hi - lo) / 15).clamp(min=1e-6)
    zero = (-lo / scale).round().clamp(0, 15)
    q = (w / scale[:, None, :] + zero[:, None, :]).round().clamp(0, 15)
    return pack_int4(q.reshape(K, N).to(torch.int32)), scale.to(weight.dtype), zero.to(weight.dtype)


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """int32 [K/8, N] -> int32 [K, N]: nibble i of each word is K index 8r + i."""
    shifts = torch.arange(0, 32, 4, dtype=torch.int32, device=packed.device).view(1, 8, 1)
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


def quantize_fp8(weight: torch.Tensor):
    """fp16 [N, K] -> (e4m3 bytes uint8 [K, N], scale fp16 [N]): per output row, scale = max |w| / 448
    clamped to >= 1e-12, then w / scale clamped to +-448 and rounded to e4m3 by torch's cast
    (kernels/fp8.py:25-30)."""
    w = weight.float()
    scale = (w.abs().amax(dim=1) / 448.0).clamp(min=1e-12)
    wq = (w / scale[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return wq.t().contiguous().view(torch.uint8), scale.to(weight.dtype)


def rmsnorm_ref(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, residual=None):
    """The reference's RMSNorm on torch (kernels/reference.py:9-19): x + residual in fp16, mean of
    squares in fp32, weight * fp16(h * rsqrt(var + eps)). Returns `out` or `(out, x + residual)`."""
    if residual is not None:
        x = x + residual
    h = x.float()
    out = weight * (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return out if residual is None else (out, x)


def swiglu_ref(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up in fp16 (kernels/reference.py:22-24)."""
    return torch.nn.functional.silu(gate) * up
