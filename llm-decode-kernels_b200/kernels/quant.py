"""4-bit weight format (same layout as the reference's kernels/quant.py:1-11).

For a linear layer with weight W of shape [N, K] (out_features, in_features):
- `qweight`: int32 [K // 8, N]; each int32 holds 8 consecutive K values of one output column,
  value i in bits 4i..4i+3 (unsigned 0..15). N is contiguous.
- `scales`, `zeros`: fp16 [K // group_size, N]. Dequantized weight: (q - zero) * scale.
Quantization is round-to-nearest, asymmetric, group size 128 along K.

Every function runs a CUDA kernel of libdecodek (bit-exact with the reference's torch code).
"""

from __future__ import annotations

import torch

from kernels import _lib

PACK = 8  # int4 values per int32 (reference kernels/quant.py:17)


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """[K, N] integers in 0..15 -> [K // 8, N] int32 (reference kernels/quant.py:20-28)."""
    K, N = q.shape
    _lib.reference_assert(K % PACK == 0, "K must be a multiple of 8")
    _lib.require_cuda("pack_int4", q)
    q = q.to(torch.int32).contiguous()
    out = torch.empty((K // PACK, N), dtype=torch.int32, device=q.device)
    _lib.call("dk_pack_int4", _lib.ptr(q), _lib.ptr(out), K, N, _lib.stream_of(q))
    return out


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """[K // 8, N] int32 -> [K, N] int32 in 0..15 (reference kernels/quant.py:31-35)."""
    _lib.require_cuda("unpack_int4", packed)
    _lib.require_dtype("unpack_int4", torch.int32, packed)
    packed = packed.contiguous()
    R, N = packed.shape
    out = torch.empty((R * PACK, N), dtype=torch.int32, device=packed.device)
    _lib.call("dk_unpack_int4", _lib.ptr(packed), _lib.ptr(out), R * PACK, N, _lib.stream_of(packed))
    return out


def quantize_rtn(weight: torch.Tensor, group_size: int = 128):
    """RTN asymmetric int4 quantization of an [N, K] fp16 weight (reference kernels/quant.py:38-49).

    Returns (qweight int32 [K/8, N], scales fp16 [K/G, N], zeros fp16 [K/G, N]), bit-exact with the
    reference."""
    N, K = weight.shape
    _lib.reference_assert(K % group_size == 0, f"K={K} must be a multiple of group_size={group_size}")
    _lib.require_cuda("quantize_rtn", weight)
    _lib.require_dtype("quantize_rtn", torch.float16, weight)
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    dev = weight.device
    qw = torch.empty((K // PACK, N), dtype=torch.int32, device=dev)
    s = torch.empty((K // group_size, N), dtype=weight.dtype, device=dev)
    z = torch.empty((K // group_size, N), dtype=weight.dtype, device=dev)
    _lib.call("dk_quantize_rtn", _lib.ptr(weight), weight.stride(0), _lib.ptr(qw), _lib.ptr(s), _lib.ptr(z),
              N, K, group_size, _lib.stream_of(weight))
    return qw, s, z


def weight_bytes(N: int, K: int, group_size: int = 128) -> int:
    """Bytes a W4A16 kernel must read for the weight: packed int4 + fp16 scales and zeros
    (reference kernels/quant.py:52-54)."""
    return N * K // 2 + 2 * (K // group_size) * N * 2
