"""FP8 e4m3 weight-only path (kernels.fp8, C-ABI dk_quantize_fp8 / dk_w8a16_matmul) vs the oracle:
quantization bit-exact, matmul within rtol 2e-2 / atol 2e-3 of the fp32 reference on the same fp8
values (reference tests: tests/test_fp8.py)."""

import numpy as np
import pytest
import torch

import oracle
from _util import MATMUL_TOL, bits16, to_cuda
from oracle import ref

pytestmark = pytest.mark.gpu


def _case(M, N, K, seed=0, bias=False):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(N, K, generator=g) * 0.02).half().numpy()
    x = torch.randn(M, K, generator=g).half().numpy()
    b = (torch.randn(N, generator=g) * 0.1).half().numpy() if bias else None
    wq, s = oracle.quantize_fp8(w)
    return x, w, wq, s, b


def _check(M, N, K, bias=False, config=None):
    from kernels.fp8 import FP8, w8a16_matmul

    x, _, wq, s, b = _case(M, N, K, bias=bias)
    xc, sc, bc = to_cuda(x, s, b)
    wc = torch.from_numpy(wq).cuda().view(FP8)
    out = w8a16_matmul(xc, wc, sc, bias=bc, config=config)
    assert out.shape == (M, N) and out.dtype == torch.float16
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.w8a16_ref(x, wq, s, b), **MATMUL_TOL)


@pytest.mark.parametrize("case", ["fp80", "fp81", "fp82", "fp8edge"])
def test_quantize_fp8_golden_bit_exact(golden, case):
    from kernels.fp8 import dequantize_fp8, quantize_fp8

    g = golden("fp8")
    (w,) = to_cuda(g[f"{case}_w"])
    wq, s = quantize_fp8(w)
    assert wq.shape == (w.shape[1], w.shape[0]) and s.shape == (w.shape[0],)
    assert np.array_equal(wq.view(torch.uint8).cpu().numpy(), g[f"{case}_wq"])
    assert np.array_equal(bits16(s), bits16(g[f"{case}_scale"]))
    assert np.array_equal(bits16(dequantize_fp8(wq, s)), bits16(g[f"{case}_deq"]))


@pytest.mark.parametrize("N,K", [(17920, 1536), (1536, 8960), (2048, 1536), (300, 200)])
def test_quantize_fp8_matches_oracle(N, K):
    from kernels.fp8 import quantize_fp8

    w = (torch.randn(N, K) * 0.02).half()
    wq, s = quantize_fp8(w.cuda())
    owq, os_ = oracle.quantize_fp8(w.numpy())
    assert np.array_equal(wq.view(torch.uint8).cpu().numpy(), owq)
    assert np.array_equal(bits16(s), bits16(os_))


def test_roundtrip_error_bound():
    """reference tests/test_fp8.py:26-34: |deq - w| <= |w|/16 + s*2^-9 + 1e-5."""
    from kernels.fp8 import dequantize_fp8, quantize_fp8

    w = (torch.randn(64, 256) * 0.02).half().cuda()
    wq, s = quantize_fp8(w)
    err = (dequantize_fp8(wq, s).float() - w.float()).abs()
    bound = w.float().abs() / 16 + s.float()[:, None] * 2**-9 + 1e-5
    assert (err <= bound).all()


CFG = dict(BLOCK_M=16, BLOCK_N=32, BLOCK_K=32, SPLIT_K=1, GROUP_M=8)


@pytest.mark.parametrize("M,N,K", [(1, 64, 128), (5, 40, 96), (17, 96, 256)])
def test_fp8_direct(M, N, K):
    _check(M, N, K, config=CFG)


def test_fp8_split_and_gemv():
    _check(2, 48, 256, config={**CFG, "SPLIT_K": 3})
    _check(1, 48, 256, bias=True, config={"GEMV": True, "BLOCK_N": 32, "BLOCK_K": 64, "SPLIT_K": 2})


@pytest.mark.parametrize("M", [1, 4, 16])
@pytest.mark.parametrize("N,K", [(17920, 1536), (1536, 8960), (2048, 1536), (151936, 1536)])
def test_fp8_decode_shapes(M, N, K):
    _check(M, N, K, bias=(N == 2048))


@pytest.mark.parametrize("split", [1, 2, 5, 8])
@pytest.mark.parametrize("block_n", [32, 64, 128, 256])
def test_fp8_every_tile_and_split(split, block_n):
    _check(3, 1536, 8960, config={"SPLIT_K": split, "BLOCK_N": block_n})
    _check(9, 512, 1000, bias=True, config={"SPLIT_K": split, "BLOCK_N": block_n})


def test_fp8_rows_split_when_staging_is_full():
    """14 rows of a K = 18944 slice: no tile fits 14 staged rows, so the rows go in launches of 7."""
    _check(14, 1536, 18944)


def test_fp8_prefill_rows():
    _check(40, 1536, 1536)


def test_fp8_golden(golden):
    from kernels.fp8 import FP8, w8a16_matmul

    g = golden("fp8")
    xc, sc, bc = to_cuda(g["w8_x"], g["w8_scale"], g["w8_bias"])
    wc = torch.from_numpy(g["w8_wq"]).cuda().view(FP8)
    out = w8a16_matmul(xc, wc, sc, bias=bc)
    np.testing.assert_allclose(out.float().cpu().numpy(), g["w8_ref"], **MATMUL_TOL)


@pytest.mark.parametrize("M,N,K,bias", [(128, 128, 64, False), (200, 208, 192, True), (256, 1536, 1536, True),
                                        (512, 17920, 1536, False), (130, 1536, 8960, False)])
def test_w8a16_tensor_core_gemm(M, N, K, bias):
    """M >= 128 runs the tcgen05 GEMM (e4m3 tile converted to fp16 in shared memory, scale on the
    fp32 accumulator): same tolerance against the oracle, deterministic, and close to the 16-row
    decode kernel (DECODE_GEMV)."""
    from kernels.fp8 import FP8, w8a16_matmul

    x, _, wq, s, b = _case(M, N, K, seed=M + K, bias=bias)
    xc, sc, bc = to_cuda(x, s, b)
    wc = torch.from_numpy(wq).cuda().view(FP8)
    out = w8a16_matmul(xc, wc, sc, bias=bc)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.w8a16_ref(x, wq, s, b), **MATMUL_TOL)
    assert torch.equal(out, w8a16_matmul(xc, wc, sc, bias=bc))
    gemv = w8a16_matmul(xc, wc, sc, bias=bc, config={"DECODE_GEMV": True})
    torch.testing.assert_close(out.float(), gemv.float(), **MATMUL_TOL)


@pytest.mark.parametrize("M", [16, 17, 32, 48, 100])
@pytest.mark.parametrize("N,K", [(2048, 1536), (1536, 8960), (256, 4096)])
def test_w8a16_small_m_tensor_core(M, N, K):
    """16..127 rows run the tcgen05 small-M kernel (e4m3 tile converted to fp16 in shared memory, batch
    rows as the MMA's N, cluster split-K): oracle tolerance, deterministic, close to the decode kernel."""
    from kernels.fp8 import FP8, w8a16_matmul

    x, _, wq, s, b = _case(M, N, K, seed=M + N, bias=True)
    xc, sc, bc = to_cuda(x, s, b)
    wc = torch.from_numpy(wq).cuda().view(FP8)
    out = w8a16_matmul(xc, wc, sc, bias=bc)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.w8a16_ref(x, wq, s, b), **MATMUL_TOL)
    assert torch.equal(out, w8a16_matmul(xc, wc, sc, bias=bc))


@pytest.mark.parametrize("M,N,K", [(20, 208, 192), (64, 1008, 64)])
def test_w8a16_small_m_edges(M, N, K):
    from kernels.fp8 import FP8, w8a16_matmul

    x, _, wq, s, b = _case(M, N, K, seed=7, bias=True)
    xc, sc, bc = to_cuda(x, s, b)
    out = w8a16_matmul(xc, torch.from_numpy(wq).cuda().view(FP8), sc, bias=bc)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.w8a16_ref(x, wq, s, b), **MATMUL_TOL)
