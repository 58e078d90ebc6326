"""W4A16 tensor-core GEMM (tcgen05 + TMEM; dk_w4a16_matmul with M >= 128 and N >= 128) vs the oracle's
dequantize-then-fp32-matmul (reference kernels/reference.py:39-45), rtol 2e-2 / atol 2e-3, and vs the
decode GEMV run over 16-row blocks. The GEMM rounds every dequantized weight to fp16 like the
reference, so the only differences are fp32 summation order and the final fp16 rounding."""

import pytest
import torch

from _util import assert_matmul_close, to_cuda, w4_case, w4_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,bias", [
    (128, 128, 128, False), (200, 200, 256, True), (256, 1536, 1536, True), (512, 2048, 1536, False),
    (130, 17920, 1536, False), (384, 1536, 8960, False), (129, 256, 4096, True), (640, 4608, 3584, True),
    # 256-column tiles (taken when the 256 x 256 tile grid has at least one tile per SM)
    (1024, 17920, 1536, True), (520, 38008, 512, False),
])
def test_gemm_matches_oracle(M, N, K, bias):
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, b = w4_case(M, N, K, seed=M + N, bias=bias)
    xc, qc, sc, zc, bc = to_cuda(x, qw, s, z, b)
    out = w4a16_matmul(xc, qc, sc, zc, 128, bias=bc)
    assert_matmul_close(out, w4_ref(x, qw, s, z, b))
    again = w4a16_matmul(xc, qc, sc, zc, 128, bias=bc)
    assert torch.equal(out, again)  # deterministic
    from kernels import _lib

    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(256, 2048, 1536), (1024, 1536, 8960)])
def test_gemm_matches_decode_gemv(M, N, K):
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, _ = w4_case(M, N, K, seed=3)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    tc = w4a16_matmul(xc, qc, sc, zc).float()
    gemv = w4a16_matmul(xc, qc, sc, zc, config={"DECODE_GEMV": True, "FACTORED": False}).float()
    torch.testing.assert_close(tc, gemv, rtol=2e-2, atol=2e-3)


def test_gemm_strided_and_3d_input():
    from kernels.w4a16 import w4a16_matmul

    M, N, K = 256, 1024, 1024
    x, qw, s, z, _ = w4_case(M, N, K, seed=5)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    wide = torch.zeros(M, K + 64, dtype=torch.float16, device="cuda")
    wide[:, :K] = xc
    out = w4a16_matmul(wide[:, :K], qc, sc, zc)  # row stride K + 64
    assert_matmul_close(out, w4_ref(x, qw, s, z, None))
    out3 = w4a16_matmul(xc.view(2, 128, K), qc, sc, zc)
    assert out3.shape == (2, 128, N) and torch.equal(out3.view(M, N), out)


def test_gemm_in_cuda_graph():
    from kernels.bench.harness import capture
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, b = w4_case(256, 2048, 1536, seed=9, bias=True)
    xc, qc, sc, zc, bc = to_cuda(x, qw, s, z, b)
    ref = w4a16_matmul(xc, qc, sc, zc, bias=bc)
    res = {}

    def step():
        res["y"] = w4a16_matmul(xc, qc, sc, zc, bias=bc)

    step()
    torch.cuda.synchronize()
    graph, _ = capture(step)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(res["y"], ref)
    del graph


def test_prefill_swiglu_and_norm_paths():
    """M >= 128 through the fused entry points runs the GEMM plus the separate kernels: same
    results as those ops called one by one."""
    from kernels.rmsnorm import rmsnorm
    from kernels.swiglu import swiglu_fused
    from kernels.w4a16 import w4a16_matmul, w4a16_rmsnorm_matmul, w4a16_swiglu

    M, I, K = 256, 1024, 1536
    x, qw, s, z, _ = w4_case(M, 2 * I, K, seed=4)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    assert torch.equal(w4a16_swiglu(xc, qc, sc, zc), swiglu_fused(w4a16_matmul(xc, qc, sc, zc)))
    r = torch.randn(M, K, device="cuda").half()
    nw = (1 + 0.05 * torch.randn(K, device="cuda")).half()
    y, res = w4a16_rmsnorm_matmul(xc, nw, 1e-6, r, qc, sc, zc, swiglu=True)
    h, res2 = rmsnorm(xc, nw, 1e-6, residual=r)
    assert torch.equal(res, res2)
    assert torch.equal(y, swiglu_fused(w4a16_matmul(h, qc, sc, zc)))


# ----------------------------------------------------------- small-M (batched decode) tensor-core path
@pytest.mark.parametrize("M", [9, 12, 16, 17, 24, 32, 40, 64, 65, 100, 127])
@pytest.mark.parametrize("N,K", [(2048, 1536), (1536, 8960), (3584, 2432), (256, 4096)])
def test_small_m_tcgen05_matches_oracle(M, N, K):
    """16 < M < 128 rows, and 9-16 rows with K >= 4096, run the swap-AB tcgen05 kernel (batch rows as
    the MMA's N, cluster split-K; the other shapes here the decode GEMV): the oracle's tolerance,
    deterministic."""
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, b = w4_case(M, N, K, seed=M * 3 + N, bias=True)
    xc, qc, sc, zc, bc = to_cuda(x, qw, s, z, b)
    out = w4a16_matmul(xc, qc, sc, zc, 128, bias=bc, config={"STATIC_WEIGHTS": True})
    assert_matmul_close(out, w4_ref(x, qw, s, z, b))
    assert torch.equal(out, w4a16_matmul(xc, qc, sc, zc, 128, bias=bc))
    from kernels import _lib

    assert _lib.device_error() == 0


def test_small_m_gate_up_and_graph():
    """A gate_up-sized layer (one CTA per 128 columns, no split) at batch 32, inside a CUDA graph."""
    from kernels.bench.harness import capture
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, _ = w4_case(32, 17920, 1536, seed=12)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    ref = w4a16_matmul(xc, qc, sc, zc)
    assert_matmul_close(ref, w4_ref(x, qw, s, z, None))
    res = {}

    def step():
        res["y"] = w4a16_matmul(xc, qc, sc, zc)

    step()
    torch.cuda.synchronize()
    graph, _ = capture(step)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(res["y"], ref)
    del graph


@pytest.mark.parametrize("M", [17, 32, 64])
def test_small_m_fused_entry_points_split(M):
    """Above 16 rows the fused SwiGLU / RMSNorm entry points run the small-M GEMM plus the separate
    kernels: identical to calling those ops one by one."""
    from kernels.rmsnorm import rmsnorm
    from kernels.swiglu import swiglu_fused
    from kernels.w4a16 import w4a16_matmul, w4a16_rmsnorm_matmul, w4a16_swiglu

    I, K = 8960, 1536
    x, qw, s, z, _ = w4_case(M, 2 * I, K, seed=M)
    xc, qc, sc, zc = to_cuda(x, qw, s, z)
    assert torch.equal(w4a16_swiglu(xc, qc, sc, zc), swiglu_fused(w4a16_matmul(xc, qc, sc, zc)))
    r = torch.randn(M, K, device="cuda").half()
    nw = (1 + 0.05 * torch.randn(K, device="cuda")).half()
    y, res = w4a16_rmsnorm_matmul(xc, nw, 1e-6, r, qc, sc, zc, swiglu=True)
    h, res2 = rmsnorm(xc, nw, 1e-6, residual=r)
    assert torch.equal(res, res2)
    assert torch.equal(y, swiglu_fused(w4a16_matmul(h, qc, sc, zc)))


@pytest.mark.parametrize("M,N,K", [(20, 200, 256), (64, 1000, 128), (33, 136, 2048), (16, 4104, 4096)])
def test_small_m_edges(M, N, K):
    """Small-M tcgen05 kernel at a partial last 128-column tile, the smallest K (one 128-group), and
    exactly 64 rows."""
    from kernels.w4a16 import w4a16_matmul

    x, qw, s, z, b = w4_case(M, N, K, seed=N + K, bias=True)
    xc, qc, sc, zc, bc = to_cuda(x, qw, s, z, b)
    assert_matmul_close(w4a16_matmul(xc, qc, sc, zc, 128, bias=bc), w4_ref(x, qw, s, z, b))
