"""Fused SwiGLU (kernels.swiglu, C-ABI dk_swiglu) vs the oracle: within 2 fp16 ulps (silu's exp
differs in the last fp32 bits between libraries, which can move the fp16 silu by one ulp before the
fp16 multiply by `up`) and within the reference's 1e-2 tolerance.
(Reference tests: tests/test_swiglu.py.)"""

import numpy as np
import pytest
import torch

from _util import ELEMWISE_TOL, bits16, to_cuda
from oracle import ref

pytestmark = pytest.mark.gpu

SMALL = [(1, 64), (3, 1000), (4, 2048)]
LARGE = [(1, 8960), (16, 8960), (2048, 8960), (333, 4097)]


def _ulps(a, b):
    a = bits16(a).astype(np.int32)
    b = bits16(b).astype(np.int32)
    a = np.where(a & 0x8000, 0x8000 - a, a)
    b = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(a - b)


def _check(M, I, seed=0):
    from kernels.swiglu import swiglu, swiglu_fused

    g = torch.Generator().manual_seed(seed)
    gate = (torch.randn(M, I, generator=g) * 3).half()
    up = torch.randn(M, I, generator=g).half()
    exp = ref.swiglu_ref(gate.numpy(), up.numpy())
    out = swiglu(gate.cuda(), up.cuda())
    assert _ulps(out, exp).max() <= 2
    np.testing.assert_allclose(out.float().cpu().numpy(), exp.astype(np.float32), **ELEMWISE_TOL)
    fused = torch.cat([gate, up], dim=-1).cuda()
    assert _ulps(swiglu_fused(fused), exp).max() <= 2


@pytest.mark.parametrize("M,I", SMALL + LARGE)
def test_swiglu(M, I):
    _check(M, I)


def test_swiglu_golden(golden):
    from kernels.swiglu import swiglu

    g = golden("norm_act")
    for i in range(4):
        gc, uc = to_cuda(g[f"swi{i}_g"], g[f"swi{i}_u"])
        assert _ulps(swiglu(gc, uc), g[f"swi{i}_out"]).max() <= 2
    gc, uc = to_cuda(g["swiedge_g"], g["swiedge_u"])
    assert _ulps(swiglu(gc, uc), g["swiedge_out"]).max() <= 2


def test_swiglu_3d():
    from kernels.swiglu import swiglu_fused

    gu = torch.randn(2, 5, 512).half()
    out = swiglu_fused(gu.cuda())
    assert out.shape == (2, 5, 256)
    exp = ref.swiglu_ref(gu[..., :256].numpy(), gu[..., 256:].numpy())
    assert _ulps(out, exp).max() <= 2


@pytest.mark.parametrize("M,N,K", [(1, 17920, 1536), (4, 2 * 8960, 1536), (16, 512, 1024), (2, 2 * 96, 256)])
def test_gate_up_with_fused_swiglu(M, N, K):
    """w4a16_swiglu (gate_up GEMV with SwiGLU in its epilogue) == swiglu_fused(w4a16_matmul(...))
    within 1 fp16 ulp: the fused epilogue rounds g and u to fp16 before the activation exactly like
    the two-kernel path, only the fp32 summation order of the GEMV differs."""
    from kernels.w4a16 import w4a16_swiglu
    from _util import w4_case, w4_ref

    x, qw, s, z, _ = w4_case(M, N, K)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    fused = w4a16_swiglu(xc, qc, sc, zc).cpu().numpy()
    gu = w4_ref(x, qw, s, z, None).astype(np.float16)
    exp = ref.swiglu_ref(gu[:, : N // 2], gu[:, N // 2:])
    np.testing.assert_allclose(fused.astype(np.float32), exp.astype(np.float32), rtol=2e-2, atol=4e-3)
