"""Argument shapes the kernels cannot check themselves (they receive raw pointers and sizes) are
checked by the Python entry points before anything reaches the device, so a smaller tensor is never
read past its end (CPU only: the checks run before the device checks). They raise ValueError, which
python -O keeps (an `assert` statement would vanish)."""

import pytest
import torch


def _w4(N=64, K=256, g=128):
    return (torch.zeros(K // 8, N, dtype=torch.int32), torch.ones(K // g, N, dtype=torch.float16),
            torch.zeros(K // g, N, dtype=torch.float16))


def test_w4a16_scales_zeros_and_bias_shapes():
    from kernels.tp import w4a16_matmul_allreduce
    from kernels.w4a16 import w4a16_matmul, w4a16_rmsnorm_matmul, w4a16_swiglu

    x = torch.zeros(1, 256, dtype=torch.float16)
    qw, s, z = _w4()
    with pytest.raises(ValueError, match="scales and zeros"):
        w4a16_matmul(x, qw, s[:1], z)
    with pytest.raises(ValueError, match="scales and zeros"):
        w4a16_swiglu(x, qw, s, z[:, :32])
    with pytest.raises(ValueError, match="bias"):
        w4a16_matmul(x, qw, s, z, bias=torch.zeros(32, dtype=torch.float16))
    with pytest.raises(ValueError, match="norm_weight"):
        w4a16_rmsnorm_matmul(x, torch.ones(128, dtype=torch.float16), 1e-6, None, qw, s, z)
    with pytest.raises(ValueError, match="residual"):
        w4a16_rmsnorm_matmul(x, torch.ones(256, dtype=torch.float16), 1e-6, torch.zeros(2, 256, dtype=torch.float16),
                             qw, s, z)
    with pytest.raises(ValueError, match="scales and zeros"):
        w4a16_matmul_allreduce(x, qw, s.t().contiguous(), z, comm=None)
    with pytest.raises(RuntimeError, match="CUDA"):  # right shapes: the next check is the device
        w4a16_matmul(x, qw, s, z)


def test_w8a16_scale_and_bias_shapes():
    from kernels.fp8 import FP8, w8a16_matmul

    x = torch.zeros(1, 64, dtype=torch.float16)
    wq = torch.zeros(64, 32, dtype=torch.uint8).view(FP8)
    with pytest.raises(ValueError, match="scale"):
        w8a16_matmul(x, wq, torch.ones(16, dtype=torch.float16))
    with pytest.raises(ValueError, match="bias"):
        w8a16_matmul(x, wq, torch.ones(32, dtype=torch.float16), bias=torch.zeros(33, dtype=torch.float16))


def test_rmsnorm_swiglu_attention_shapes():
    from kernels.attention import decode_attention
    from kernels.rmsnorm import rmsnorm
    from kernels.swiglu import swiglu

    x = torch.zeros(2, 8, dtype=torch.float16)
    with pytest.raises(ValueError, match="weight"):
        rmsnorm(x, torch.ones(4, dtype=torch.float16))
    with pytest.raises(ValueError, match="residual"):
        rmsnorm(x, torch.ones(8, dtype=torch.float16), residual=torch.zeros(1, 8, dtype=torch.float16))
    with pytest.raises(ValueError, match="same shape"):
        swiglu(torch.zeros(2, 8, dtype=torch.float16), torch.zeros(3, 8, dtype=torch.float16))
    B, nq, nkv, L, hd = 2, 4, 2, 16, 32
    qkv = torch.zeros(B, 1, (nq + 2 * nkv) * hd, dtype=torch.float16)
    small = torch.zeros(1, nkv, L, hd, dtype=torch.float16)  # one sequence's cache for a batch of 2
    pos = torch.zeros(1, dtype=torch.int64)
    rope = torch.zeros(1, hd, dtype=torch.float16)
    with pytest.raises(ValueError, match="k_cache and v_cache"):
        decode_attention(qkv, small, small, pos, rope, rope, nq, nkv)
