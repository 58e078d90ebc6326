"""The M <= 16 decode entry point (kernels.cuda.w4a16_cuda.w4a16_decode_cuda) vs the oracle.
Same cases as the reference's tests/test_w4a16_cuda.py, at the BASELINE tolerance."""

import pytest
import torch

from _util import assert_matmul_close, to_cuda, w4_case, w4_ref

pytestmark = pytest.mark.gpu


def _check(M, N, K, split=None, bias=False):
    from kernels.cuda.w4a16_cuda import w4a16_decode_cuda

    x, qw, s, z, b = w4_case(M, N, K, bias=bias)
    xc, qc, sc, zc, bc = to_cuda(x, qw, s, z, b)
    out = w4a16_decode_cuda(xc, qc, sc, zc, bias=bc, split_k=split)
    assert out.shape == (M, N) and out.dtype == torch.float16
    assert_matmul_close(out, w4_ref(x, qw, s, z, b))


@pytest.mark.parametrize("M", [1, 2, 3, 4, 7, 8, 16])
@pytest.mark.parametrize("split", [1, 4])
def test_cuda_decode_qwen(M, split):
    _check(M, 1536, 1536, split)


@pytest.mark.parametrize("N,K", [(2048, 1536), (17920, 1536), (1536, 8960), (4096, 14336)])
def test_cuda_decode_autosplit(N, K):
    _check(1, N, K)
    _check(16, N, K)


def test_cuda_odd_n_and_bias():
    _check(5, 1000, 1024, split=3, bias=True)  # N not a multiple of 128
    _check(1, 132, 256, split=1, bias=True)


def test_cuda_split_16_clamps():
    _check(2, 1536, 8960, split=16)


def test_cuda_rejects_large_m():
    with pytest.raises(RuntimeError):
        _check(17, 128, 128, split=1)
