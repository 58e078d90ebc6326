"""The decode (M <= 16) W4A16 entry point (reference kernels/cuda/w4a16_cuda.py:45-56).

The reference JIT-builds a CUDA-core kernel for sm_89/sm_90 and times split-K factors 1..16 per
shape. Here the same contract runs libdecodek's sm_100a decode kernel (tensor-core dot products,
bulk-copy weight streaming, cluster split-K); `split_k` maps to the cluster split (1..8, larger
requests are clamped to 8), None lets the cost model choose. Like the reference, M > 16 raises
RuntimeError and N must be a multiple of 4.
"""

from __future__ import annotations

from kernels.w4a16 import w4a16_matmul

_split_choice: dict[tuple, int] = {}


def w4a16_decode_cuda(x, qweight, scales, zeros, group_size=128, bias=None, split_k=None):
    """y = x @ dequant(W).T for M <= 16 rows. Same contract as kernels.w4a16.w4a16_matmul."""
    K = x.shape[-1]
    N = qweight.shape[1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    if not 1 <= M <= 16:
        raise RuntimeError("decode kernel supports M <= 16")
    if N % 4 != 0:
        raise RuntimeError("N must be a multiple of 4 (16-byte loads)")
    if qweight.shape[0] * 8 != K or K % group_size != 0 or group_size % 8 != 0:
        raise RuntimeError("w4a16_decode_cuda: need qweight.shape[0]*8 == K and K % group_size == 0")
    cfg = None if split_k is None else {"SPLIT_K": max(1, min(int(split_k), 8))}
    key = (min(1 << (M - 1).bit_length(), 16), N, K, bias is not None)
    _split_choice.setdefault(key, split_k or 0)
    out = w4a16_matmul(x2, qweight, scales, zeros, group_size, bias=bias, config=cfg)
    return out.view(*x.shape[:-1], N)


def split_choices() -> dict:
    return {str(k): v for k, v in _split_choice.items()}


def export_choices() -> dict:
    return {",".join(map(str, k)): v for k, v in _split_choice.items()}


def import_choices(choices: dict) -> None:
    for k, v in choices.items():
        m, n, kk, b = k.split(",")
        _split_choice[(int(m), int(n), int(kk), b == "True")] = v
