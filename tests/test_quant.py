"""int4 format kernels vs the oracle and the reference's golden vectors: bit-exact.
(Reference tests: tests/test_quant.py.)"""

import numpy as np
import pytest
import torch

import oracle
from _util import bits16, to_cuda

pytestmark = pytest.mark.gpu


def test_pack_roundtrip_golden(golden):
    from kernels.quant import pack_int4, unpack_int4

    g = golden("quant")
    (q,) = to_cuda(g["pack_q"])
    packed = pack_int4(q)
    assert packed.shape == (8, 24) and packed.dtype == torch.int32
    assert np.array_equal(packed.cpu().numpy(), g["pack_packed"])
    assert torch.equal(unpack_int4(packed), q)


def test_pack_extremes():
    """all 15 -> int32 -1 (reference tests/test_quant.py:15-18)."""
    from kernels.quant import pack_int4, unpack_int4

    q = torch.full((16, 3), 15, dtype=torch.int32, device="cuda")
    assert torch.equal(pack_int4(q), torch.full((2, 3), -1, dtype=torch.int32, device="cuda"))
    assert torch.equal(unpack_int4(pack_int4(q)), q)


def test_pack_matches_oracle_random_ints():
    """Values outside 0..15 too: the packing wraps exactly like the reference's int64 math."""
    from kernels.quant import pack_int4

    q = np.random.randint(-40, 40, size=(256, 40)).astype(np.int32)
    assert np.array_equal(pack_int4(torch.from_numpy(q).cuda()).cpu().numpy(), oracle.pack_int4(q))


@pytest.mark.parametrize("case", ["rtn0", "rtn1", "rtn2", "rtn3", "rtn4", "rtnedge"])
def test_quantize_rtn_golden_bit_exact(golden, case):
    from kernels.quant import quantize_rtn

    g = golden("quant")
    (w,) = to_cuda(g[f"{case}_w"])
    qw, s, z = quantize_rtn(w, 128)
    assert np.array_equal(qw.cpu().numpy(), g[f"{case}_qweight"])
    assert np.array_equal(bits16(s), bits16(g[f"{case}_scales"]))
    assert np.array_equal(bits16(z), bits16(g[f"{case}_zeros"]))


@pytest.mark.parametrize("N,K,G", [(2048, 1536, 128), (17920, 1536, 128), (1536, 8960, 128),
                                   (96, 512, 64), (40, 256, 256), (8, 64, 8)])
def test_quantize_rtn_matches_oracle(N, K, G):
    from kernels.quant import quantize_rtn

    w = (torch.randn(N, K) * 0.02).half()
    qw, s, z = quantize_rtn(w.cuda(), G)
    oq, os_, oz = oracle.quantize_rtn(w.numpy(), G)
    assert np.array_equal(qw.cpu().numpy(), oq)
    assert np.array_equal(bits16(s), bits16(os_))
    assert np.array_equal(bits16(z), bits16(oz))


def test_quantize_rtn_strided_input():
    from kernels.quant import quantize_rtn

    big = (torch.randn(64, 512) * 0.02).half()
    w = big[:, :256]  # row stride 512
    qw, s, z = quantize_rtn(w.cuda(), 128)
    oq, os_, oz = oracle.quantize_rtn(w.contiguous().numpy(), 128)
    assert np.array_equal(qw.cpu().numpy(), oq) and np.array_equal(bits16(s), bits16(os_))


def test_dequantize_bit_exact(golden):
    from kernels.reference import dequantize_ref

    g = golden("matmul")
    for i in range(len(g["w4_cases"])):
        if f"w4_{i}_deq" not in g:
            continue
        qw, s, z = to_cuda(g[f"w4_{i}_qweight"], g[f"w4_{i}_scales"], g[f"w4_{i}_zeros"])
        assert np.array_equal(bits16(dequantize_ref(qw, s, z, 128)), bits16(g[f"w4_{i}_deq"]))


def test_weight_bytes(golden):
    from kernels.quant import weight_bytes

    assert weight_bytes(1536, 1536) == 1536 * 1536 // 2 + 2 * 12 * 1536 * 2
    shapes = [(1536, 1536), (2048, 1536), (17920, 1536), (1536, 8960), (151936, 1536)]
    assert [weight_bytes(n, k) for n, k in shapes] == list(golden("quant")["weight_bytes"])


def test_cpu_tensor_raises():
    from kernels.quant import quantize_rtn

    with pytest.raises(RuntimeError, match="CUDA"):
        quantize_rtn((torch.randn(8, 128) * 0.02).half(), 128)
