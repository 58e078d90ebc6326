"""W4A16 matmul (kernels.w4a16.w4a16_matmul, C-ABI dk_w4a16_matmul) vs the oracle's
dequantize-then-fp32-matmul. Tolerance rtol 2e-2 / atol 2e-3; the kernel
dequantizes with the reference's fp16 rounding, so the observed error is only fp32 summation order
plus the final fp16 rounding. (Reference tests: tests/test_w4a16.py.)"""

import numpy as np
import pytest
import torch

from _util import assert_matmul_close, to_cuda, w4_case, w4_ref

pytestmark = pytest.mark.gpu


def _check(M, N, K, bias=False, config=None, seed=0, group=128):
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, b = w4_case(M, N, K, seed=seed, bias=bias, group=group)
    xc, qc, sc, zc, bc = to_cuda(x, qw, s, z, b)
    out = w4a16_matmul(xc, qc, sc, zc, group, bias=bc, config=config)
    assert out.shape == (M, N) and out.dtype == torch.float16
    assert_matmul_close(out, w4_ref(x, qw, s, z, b, group))
    return out


def test_golden_cases(golden):
    from kernels.w4a16 import w4a16_matmul

    g = golden("matmul")
    for i, (M, N, K, has_bias) in enumerate(g["w4_cases"]):
        x, qw, s, z = to_cuda(*(g[f"w4_{i}_{k}"] for k in ("x", "qweight", "scales", "zeros")))
        (b,) = to_cuda(g[f"w4_{i}_bias"] if has_bias else None)
        out = w4a16_matmul(x, qw, s, z, 128, bias=b)
        assert out.shape == (M, N)
        assert_matmul_close(out, g[f"w4_{i}_ref"])


# Reference direct/split/gemv config dicts are accepted; SPLIT_K maps to the cluster split.
CFG = dict(BLOCK_M=16, BLOCK_N=32, BLOCK_K=64, SPLIT_K=1, GROUP_M=8)


@pytest.mark.parametrize("M,N,K", [(1, 64, 256), (3, 40, 128), (17, 96, 384)])
def test_direct_small(M, N, K):
    _check(M, N, K, config=CFG)


@pytest.mark.parametrize("split", [2, 3])
def test_split_k_small(split):
    _check(2, 48, 512, config={**CFG, "SPLIT_K": split})


def test_bias_both_paths():
    _check(1, 64, 256, bias=True, config=CFG)
    _check(1, 64, 256, bias=True, config={**CFG, "SPLIT_K": 2})


@pytest.mark.parametrize("N,K", [(64, 256), (40, 384), (96, 128)])
@pytest.mark.parametrize("split", [1, 3])
def test_gemv(N, K, split):
    _check(1, N, K, config=dict(GEMV=True, BLOCK_N=32, BLOCK_K=64, SPLIT_K=split))


def test_3d_input():
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, _ = w4_case(6, 32, 128)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    out = w4a16_matmul(xc.view(2, 3, 128), qc, sc, zc, config=CFG)
    assert out.shape == (2, 3, 32)
    assert_matmul_close(out.view(6, 32), w4_ref(x, qw, s, z, None))


QWEN = [(2048, 1536), (1536, 1536), (17920, 1536), (1536, 8960), (256, 1536), (8960, 1536)]


@pytest.mark.parametrize("M", [1, 2, 3, 4, 7, 8, 16])
@pytest.mark.parametrize("N,K", QWEN)
def test_decode_qwen_shapes(M, N, K):
    _check(M, N, K, bias=(N == 2048))


@pytest.mark.parametrize("split", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("block_n", [32, 64, 128, 256])
@pytest.mark.parametrize("exact", [False, True])
def test_every_tile_and_split(split, block_n, exact):
    cfg = {"SPLIT_K": split, "BLOCK_N": block_n, "EXACT": exact}
    _check(4, 1536, 8960, config=cfg)
    _check(16, 1000, 1024, bias=True, config=cfg)
    _check(1, 4096, 512, config=cfg)


def _ulps16(a, b):
    a = np.ascontiguousarray(a, dtype=np.float16).view(np.uint16).astype(np.int32)
    b = np.ascontiguousarray(b, dtype=np.float16).view(np.uint16).astype(np.int32)
    a = np.where(a & 0x8000, 0x8000 - a, a)
    b = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(a - b)


@pytest.mark.parametrize("M,N,K", [(1, 2048, 1536), (5, 1536, 8960), (16, 17920, 1536)])
def test_exact_dequant_rounds_like_reference(M, N, K):
    """With EXACT the kernel dequantizes with the reference's fp16 rounding, so the only
    difference left is the fp32 summation order: the fp16 output is within one ulp of the
    reference's fp32 result rounded to fp16, or within 2e-5 absolute where cancellation makes
    the output so small that an ulp is below the summation-order noise."""
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, b = w4_case(M, N, K, bias=True)
    xc, qc, sc, zc, bc = to_cuda(x, qw, s, z, b)
    out = w4a16_matmul(xc, qc, sc, zc, bias=bc, config={"EXACT": True}).cpu().numpy()
    ref32 = w4_ref(x, qw, s, z, b)
    ref = ref32.astype(np.float16)
    close = np.abs(out.astype(np.float32) - ref32) <= 2e-5
    assert ((_ulps16(out, ref) <= 1) | close).all()


def test_lm_head_m1():
    _check(1, 151936, 1536)


@pytest.mark.parametrize("M", [33, 128])
@pytest.mark.parametrize("N,K", [(1536, 1536), (8960, 1536)])
def test_prefill_sizes(M, N, K):
    _check(M, N, K)


def test_odd_shapes_and_bias():
    """reference tests/test_w4a16.py:100-103 plus N not a multiple of 8 (generic kernel)."""
    _check(3, 1000, 1024, bias=True)
    _check(100, 200, 640, bias=True)
    _check(1, 132, 256, bias=True)
    _check(5, 36, 256, bias=True)


def test_group_sizes():
    _check(2, 128, 512, group=256)
    _check(2, 128, 512, group=64)  # generic kernel (group not a multiple of 128)


def test_generic_kernel_matches():
    _check(4, 256, 512, bias=True, config={"GENERIC": True})


def test_strided_x_and_static_flag():
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, b = w4_case(4, 512, 1024, bias=True)
    big = np.zeros((4, 2048), dtype=np.float16)
    big[:, :1024] = x
    xc, qc, sc, zc, bc = to_cuda(big, qw, s, z, b)
    out = w4a16_matmul(xc[:, :1024], qc, sc, zc, bias=bc, config={"STATIC_WEIGHTS": True})
    assert_matmul_close(out, w4_ref(x, qw, s, z, b))


@pytest.mark.parametrize("config", [None, {"BLOCK_N": 32, "SPLIT_K": 1}, {"BLOCK_N": 64, "SPLIT_K": 1}])
def test_long_k_slice(config):
    """K = 32512 in one slice: staging x leaves shared memory for a two-stage ring only, fewer stages
    than the warps that share a 32- or 64-column chunk, so those forced tiles are refused and the
    automatic choice (a ring at least as deep) runs instead."""
    _check(1, 1536, 32512, config=config)


def test_rows_split_when_staging_is_full():
    """13 rows of a K = 18944 slice (Qwen2.5-7B down): the staged x of 13 rows leaves no tile, so the
    rows go in launches of 7 and 6 (before this, no tile fitted and the call failed)."""
    _check(13, 3584, 18944)


def test_deterministic():
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, _ = w4_case(8, 1536, 8960)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    a = w4a16_matmul(xc, qc, sc, zc, config={"SPLIT_K": 7})
    for _ in range(3):
        assert torch.equal(a, w4a16_matmul(xc, qc, sc, zc, config={"SPLIT_K": 7}))


def test_zero_rows_and_errors():
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, _ = w4_case(1, 64, 256)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    assert w4a16_matmul(xc[:0], qc, sc, zc).shape == (0, 64)
    with pytest.raises(AssertionError):
        w4a16_matmul(xc[:, :128], qc, sc, zc)  # K mismatch: same assert as the reference
    with pytest.raises(RuntimeError):
        w4a16_matmul(xc.float(), qc, sc, zc)


def test_no_device_errors_recorded():
    from kernels import _lib

    _check(16, 17920, 1536)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,N,K,bn", [(4, 151936, 1536, 0), (16, 40000, 1024, 256), (1, 9472, 3584, 256),
                                      (3, 2368 * 32, 512, 128)])
def test_tail_tiles(M, N, K, bn):
    """Column counts that leave some persistent CTAs a partial last tile (fewer chunks than the tile
    holds), with M <= 8 and M = 16 variants."""
    _check(M, N, K, config={"BLOCK_N": bn} if bn else None)
