"""Helpers shared by the parity tests: seeded inputs in the reference's distributions, oracle
results, and the comparison tolerances."""

from __future__ import annotations

import numpy as np
import torch

import oracle
from oracle import ref

# matmul outputs within rtol 2e-2 / atol 2e-3 of the reference
# dequantize-then-matmul in fp16 (the reference's own tests use 1e-2 / 1e-2).
MATMUL_TOL = dict(rtol=2e-2, atol=2e-3)
# fp16 elementwise outputs: the reference's tolerance (tests/test_rmsnorm.py:13, test_swiglu.py:9)
ELEMWISE_TOL = dict(rtol=1e-2, atol=1e-2)


def w4_case(M, N, K, seed=0, bias=False, group=128):
    """x ~ N(0,1) fp16 [M,K]; W ~ N(0, 0.02) fp16 [N,K] RTN-quantized by the oracle; bias 0.1*N(0,1)
    (tests/test_w4a16.py:18-23 of the reference)."""
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * 0.02).half().numpy()
    x = torch.randn(M, K, generator=g).half().numpy()
    b = (torch.randn(N, generator=g) * 0.1).half().numpy() if bias else None
    qw, s, z = oracle.quantize_rtn(w, group)
    return x, qw, s, z, b


def to_cuda(*arrs):
    return [None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def w4_ref(x, qw, s, z, b, group=128):
    return ref.w4a16_ref(x, qw, s, z, group, b)


def assert_matmul_close(out: torch.Tensor, ref32: np.ndarray, tol=MATMUL_TOL):
    assert out.dtype == torch.float16
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, ref32, **tol)


def bits16(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float16).view(np.uint16)
