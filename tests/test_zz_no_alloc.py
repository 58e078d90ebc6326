"""The allocation-free entry point dk_w4a16_matmul_reduce_static, called through the C ABI.

It exists for callers that cannot allocate device memory (a plugin inside a serving process that owns
the CUDA allocator, a runtime that forbids raw cudaMalloc): it runs the fused matmul + reduce kernel
on one GPU with its scratch in a fixed array inside the library instead of a buffer from
dk_tp_buffer_alloc. Its output must be the existing entry point's - dk_w4a16_matmul_allreduce with a
one-rank communicator - within the matmul tolerance (rtol 2e-2 / atol 2e-3), on two calls in a row
(the second call reuses the array the first one left behind).

This file is named to be collected last, so a run that stops at the first failure has run every
other test first. It passes alone in a fresh process and after the rest of the suite.
"""

import ctypes

import pytest
import torch

from _util import MATMUL_TOL

pytestmark = pytest.mark.gpu


def _layer(M, N, K, seed):
    from kernels.quant import quantize_rtn

    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * 0.02).half().cuda()
    x = torch.randn(M, K, generator=g).half().cuda()
    b = (torch.randn(N, generator=g) * 0.1).half().cuda()
    qw, s, z = quantize_rtn(w, 128)
    return x, qw, s, z, b


def _static_call(x, qw, s, z, b, y, cfg=None):
    from kernels import _lib

    M, K = x.shape
    N = qw.shape[1]
    c = _lib.MatmulConfig() if cfg is None else cfg
    return _lib.lib().dk_w4a16_matmul_reduce_static(
        _lib.ptr(x), x.stride(0), _lib.ptr(qw), _lib.ptr(s), _lib.ptr(z), _lib.ptr(b), _lib.ptr(y), y.stride(0),
        M, N, K, 128, ctypes.byref(c), _lib.stream_of(x))


@pytest.mark.parametrize("M,N,K,split", [(1, 3584, 2432, 0), (4, 2048, 1024, 0), (16, 1536, 8960, 0),
                                         (20, 1536, 1536, 0), (1, 1024, 8192, 4), (3, 8192, 512, 0)])
def test_static_matches_allreduce_entry_point(M, N, K, split):
    from kernels import _lib
    from kernels.tp import TPComm, w4a16_matmul_allreduce

    x, qw, s, z, b = _layer(M, N, K, seed=M * 7 + N)
    cfg = _lib.MatmulConfig()
    cfg.split_k = split
    comm = TPComm(max_n=8192)  # the existing entry point: a one-rank communicator from dk_tp_buffer_alloc
    try:
        ref = w4a16_matmul_allreduce(x, qw, s, z, comm, bias=b, config={"SPLIT_K": split} if split else None)
    finally:
        comm.close()
    for _ in range(2):  # two calls in a row on the shared static scratch
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        _lib.check(_static_call(x, qw, s, z, b, y, cfg), "dk_w4a16_matmul_reduce_static")
        torch.cuda.synchronize()
        torch.testing.assert_close(y.float(), ref.float(), **MATMUL_TOL)
    assert _lib.device_error() == 0


def test_static_rejects_columns_beyond_the_scratch():
    from kernels import _lib

    x, qw, s, z, b = _layer(1, 8200, 128, seed=1)
    y = torch.empty(1, 8200, dtype=torch.float16, device="cuda")
    assert _static_call(x, qw, s, z, b, y) == -1  # DK_ERR_INVALID
    assert b"8192" in _lib.lib().dk_last_error()
