"""Fused RMSNorm (kernels.rmsnorm.rmsnorm, C-ABI dk_rmsnorm) vs the oracle: the residual output
must be bit-exact (same fp16 add, reference tests/test_rmsnorm.py:30), the normalized output
within 2 fp16 ulps of the oracle (same rounding steps; the fp32 sum order differs, which can move
the normalized value by one ulp before the fp16 multiply by the weight) and within the reference's
1e-2 tolerance."""

import numpy as np
import pytest
import torch

from _util import ELEMWISE_TOL, bits16, to_cuda
from oracle import ref

pytestmark = pytest.mark.gpu

SMALL = [(1, 128), (3, 1000), (5, 1536)]
LARGE = [(1, 1536), (16, 1536), (2048, 1536), (16, 4096), (4096, 1536), (2048, 8192), (7, 8960)]


def _inputs(M, N, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, N, generator=g).half().numpy()
    r = torch.randn(M, N, generator=g).half().numpy()
    w = (1 + 0.05 * torch.randn(N, generator=g)).half().numpy()
    return x, r, w


def _ulps(a, b):
    a = bits16(a).astype(np.int32)
    b = bits16(b).astype(np.int32)
    a = np.where(a & 0x8000, 0x8000 - a, a)
    b = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(a - b)


def _check(M, N):
    from kernels.rmsnorm import rmsnorm

    x, r, w = _inputs(M, N)
    xc, rc, wc = to_cuda(x, r, w)
    out = rmsnorm(xc, wc, 1e-6)
    o_ref = ref.rmsnorm_ref(x, w, 1e-6)
    assert _ulps(out, o_ref).max() <= 2
    np.testing.assert_allclose(out.float().cpu().numpy(), o_ref.astype(np.float32), **ELEMWISE_TOL)
    out, res = rmsnorm(xc, wc, 1e-6, residual=rc)
    o_ref, r_ref = ref.rmsnorm_ref(x, w, 1e-6, residual=r)
    assert np.array_equal(bits16(res), bits16(r_ref))
    assert _ulps(out, o_ref).max() <= 2


@pytest.mark.parametrize("M,N", SMALL + LARGE)
def test_rmsnorm(M, N):
    _check(M, N)


def test_rmsnorm_golden(golden):
    from kernels.rmsnorm import rmsnorm

    g = golden("norm_act")
    for i in range(4):
        x, r, w = to_cuda(g[f"rms{i}_x"], g[f"rms{i}_r"], g[f"rms{i}_w"])
        assert _ulps(rmsnorm(x, w, 1e-6), g[f"rms{i}_out"]).max() <= 2
        out, res = rmsnorm(x, w, 1e-6, residual=r)
        assert np.array_equal(bits16(res), bits16(g[f"rms{i}_res"]))
        assert _ulps(out, g[f"rms{i}_out_res"]).max() <= 2


def test_rmsnorm_3d_input():
    from kernels.rmsnorm import rmsnorm

    x = torch.randn(2, 3, 256).half()
    w = torch.ones(256).half()
    out = rmsnorm(x.cuda(), w.cuda())
    assert out.shape == (2, 3, 256)
    assert _ulps(out, ref.rmsnorm_ref(x.numpy(), w.numpy())).max() <= 2


def test_rmsnorm_strided_rows():
    from kernels.rmsnorm import rmsnorm

    x, r, w = _inputs(4, 1536)
    big = np.zeros((4, 2048), dtype=np.float16)
    big[:, 8:1544] = x  # row stride 2048, offset 16 bytes
    bc, rc, wc = to_cuda(big, r, w)
    out, res = rmsnorm(bc[:, 8:1544], wc, 1e-6, residual=rc)
    o_ref, r_ref = ref.rmsnorm_ref(x, w, 1e-6, residual=r)
    assert np.array_equal(bits16(res), bits16(r_ref))
    assert _ulps(out, o_ref).max() <= 2


@pytest.mark.parametrize("M,N,K,swiglu,with_res", [(1, 2048, 1536, False, True), (1, 2048, 1536, False, False),
                                                   (4, 17920, 1536, True, True), (16, 1536, 8960, False, True),
                                                   (3, 512, 1024, True, False)])
def test_rmsnorm_fused_into_matmul(M, N, K, swiglu, with_res):
    """w4a16_rmsnorm_matmul == the two-kernel path rmsnorm -> w4a16_matmul / w4a16_swiglu: the new
    residual bit-exactly, the projection within the matmul tolerance of the oracle computed on the
    oracle's normalized activations."""
    from kernels.w4a16 import w4a16_rmsnorm_matmul
    from _util import MATMUL_TOL, w4_case, w4_ref

    x, r, w = _inputs(M, K, seed=7)
    _, qw, s, z, b = w4_case(M, N, K, bias=not swiglu)
    xc, rc, wc, qc, sc, zc, bc = to_cuda(x, r, w, qw, s, z, b)
    # FUSED_NORM: the single kernel at every row count here (by default only up to 2 rows)
    y, res = w4a16_rmsnorm_matmul(xc, wc, 1e-6, rc if with_res else None, qc, sc, zc, bias=bc, swiglu=swiglu,
                                  config={"FUSED_NORM": True})
    if with_res:
        xn, r_ref = ref.rmsnorm_ref(x, w, 1e-6, residual=r)
        assert np.array_equal(bits16(res), bits16(r_ref))
    else:
        xn = ref.rmsnorm_ref(x, w, 1e-6)
        assert res is None
    yr = w4_ref(xn, qw, s, z, b)
    if swiglu:
        yr16 = yr.astype(np.float16)
        yr = ref.swiglu_ref(yr16[:, : N // 2], yr16[:, N // 2:]).astype(np.float32)
        np.testing.assert_allclose(y.float().cpu().numpy(), yr, rtol=2e-2, atol=4e-3)
    else:
        np.testing.assert_allclose(y.float().cpu().numpy(), yr, **MATMUL_TOL)
