"""The allocation-free entry point dk_w4a16_matmul_reduce_static, called through the C ABI.

Some callers cannot allocate device memory: a plugin loaded into a serving process that owns the
CUDA allocator and hands the plugin only its input and output buffers, or a runtime that forbids raw
cudaMalloc (it synchronizes the device and fragments the pool the runtime manages). The entry point
runs the fused matmul + reduce kernel on one GPU with its scratch in a fixed array inside the library
instead of a buffer from dk_tp_buffer_alloc.

Each case makes two calls in a row on different inputs (different x, weights and bias), so the
second call finds the array as the first one left it. Every call's output must match the
existing entry point (dk_w4a16_matmul_allreduce with a one-rank communicator) on the same inputs
and the CPU oracle (the reference's dequantize-then-matmul), within the matmul tolerance
(rtol 2e-2 / atol 2e-3). A kernel that returned cells of the previous call would fail both
comparisons.

This file is named to be collected last, so a run that stops at the first failure has run every
other test first. It passes alone in a fresh process and after the rest of the suite.
"""

import ctypes

import numpy as np
import pytest
import torch

from _util import MATMUL_TOL, to_cuda, w4_case, w4_ref

pytestmark = pytest.mark.gpu


def _static_call(x, qw, s, z, b, y, cfg=None):
    from kernels import _lib

    M, K = x.shape
    N = qw.shape[1]
    c = _lib.MatmulConfig() if cfg is None else cfg
    return _lib.lib().dk_w4a16_matmul_reduce_static(
        _lib.ptr(x), x.stride(0), _lib.ptr(qw), _lib.ptr(s), _lib.ptr(z), _lib.ptr(b), _lib.ptr(y), y.stride(0),
        M, N, K, 128, ctypes.byref(c), _lib.stream_of(x))


# (13, 3584, 18944): the Qwen2.5-7B down projection at 13 rows, whose staged x leaves no tile at 13
# rows per launch, so the call runs fewer rows per launch
@pytest.mark.parametrize("M,N,K,split", [(1, 3584, 2432, 0), (4, 2048, 1024, 0), (16, 1536, 8960, 0),
                                         (20, 1536, 1536, 0), (1, 1024, 8192, 4), (3, 8192, 512, 0),
                                         (13, 3584, 18944, 0)])
def test_static_matches_allreduce_entry_point_and_oracle(M, N, K, split):
    from kernels import _lib
    from kernels.tp import TPComm, w4a16_matmul_allreduce

    cfg = _lib.MatmulConfig()
    cfg.split_k = split
    comm = TPComm(max_n=8192)  # the existing entry point: a one-rank communicator from dk_tp_buffer_alloc
    try:
        for call in range(2):  # two calls in a row on the shared static scratch, different inputs
            x, qw, s, z, b = w4_case(M, N, K, seed=1000 * call + M * 7 + N, bias=True)
            expect = w4_ref(x, qw, s, z, b)
            xd, qd, sd, zd, bd = to_cuda(x, qw, s, z, b)
            ref = w4a16_matmul_allreduce(xd, qd, sd, zd, comm, bias=bd,
                                         config={"SPLIT_K": split} if split else None)
            y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
            _lib.check(_static_call(xd, qd, sd, zd, bd, y, cfg), "dk_w4a16_matmul_reduce_static")
            torch.cuda.synchronize()
            got = y.float().cpu().numpy()
            np.testing.assert_allclose(got, expect, **MATMUL_TOL)
            torch.testing.assert_close(y.float(), ref.float(), **MATMUL_TOL)
    finally:
        comm.close()
    assert _lib.device_error() == 0


def test_static_rejects_columns_beyond_the_scratch():
    from kernels import _lib

    x, qw, s, z, b = to_cuda(*w4_case(1, 8200, 128, seed=1, bias=True))
    y = torch.empty(1, 8200, dtype=torch.float16, device="cuda")
    assert _static_call(x, qw, s, z, b, y) == -1  # DK_ERR_INVALID
    assert b"8192" in _lib.lib().dk_last_error()
