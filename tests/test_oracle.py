"""Pins the CPU oracle to the reference: every golden vector from the reference's own code
(`tests/golden/make_golden.py`) must be reproduced. Integer/byte outputs bit-exact; float outputs
within one fp16 ulp (numpy and torch sum in different orders)."""

import numpy as np
import pytest

import oracle
from oracle import ref


def _bits16(a):
    return np.asarray(a, dtype=np.float16).view(np.uint16)


def test_pack_roundtrip_golden(golden):
    g = golden("quant")
    assert np.array_equal(oracle.pack_int4(g["pack_q"]), g["pack_packed"])
    assert np.array_equal(oracle.unpack_int4(g["pack_packed"]), g["pack_unpacked"])
    assert np.array_equal(g["pack_unpacked"], g["pack_q"])


def test_pack_all_15_is_minus_one(golden):
    """tests/test_quant.py:15-18 of the reference: all-15 packs to int32 -1."""
    g = golden("quant")
    packed = oracle.pack_int4(np.full((16, 3), 15, dtype=np.int32))
    assert np.array_equal(packed, g["pack15_packed"])
    assert (packed == -1).all()


@pytest.mark.parametrize("case", ["rtn0", "rtn1", "rtn2", "rtn3", "rtn4", "rtnedge"])
def test_quantize_rtn_bit_exact(golden, case):
    g = golden("quant")
    qw, s, z = oracle.quantize_rtn(g[f"{case}_w"], 128)
    assert np.array_equal(qw, g[f"{case}_qweight"])
    assert np.array_equal(_bits16(s), _bits16(g[f"{case}_scales"]))
    assert np.array_equal(_bits16(z), _bits16(g[f"{case}_zeros"]))


def test_weight_bytes(golden):
    g = golden("quant")
    shapes = [(1536, 1536), (2048, 1536), (17920, 1536), (1536, 8960), (151936, 1536)]
    assert [oracle.weight_bytes(n, k) for n, k in shapes] == list(g["weight_bytes"])


def test_rtn_error_bound():
    """tests/test_quant.py:21-31 of the reference: |deq - w| <= step/2 + 1e-3."""
    w = (np.random.randn(40, 384) * 0.02).astype(np.float16)
    qw, s, z = oracle.quantize_rtn(w, 128)
    deq = oracle.dequantize_int4(qw, s, z, 128).astype(np.float32)
    step = np.repeat(s.astype(np.float32), 128, axis=0).T
    assert (np.abs(deq - w.astype(np.float32)) <= 0.5 * step + 1e-3).all()


def test_matmul_golden(golden):
    g = golden("matmul")
    for i, (M, N, K, has_bias) in enumerate(g["w4_cases"]):
        args = [g[f"w4_{i}_{k}"] for k in ("x", "qweight", "scales", "zeros")]
        if f"w4_{i}_deq" in g:
            deq = oracle.dequantize_int4(*args[1:], 128)
            assert np.array_equal(_bits16(deq), _bits16(g[f"w4_{i}_deq"]))
        bias = g[f"w4_{i}_bias"] if has_bias else None
        out = ref.w4a16_ref(*args, 128, bias)
        assert out.shape == (M, N)
        np.testing.assert_allclose(out, g[f"w4_{i}_ref"], rtol=1e-5, atol=1e-5)


def _fp16_ulps(a, b):
    a = _bits16(a).astype(np.int32)
    b = _bits16(b).astype(np.int32)
    # map sign-magnitude to a monotonic integer line
    a = np.where(a & 0x8000, 0x8000 - a, a)
    b = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(a - b)


@pytest.mark.parametrize("i", range(4))
def test_rmsnorm_golden(golden, i):
    g = golden("norm_act")
    x, r, w = g[f"rms{i}_x"], g[f"rms{i}_r"], g[f"rms{i}_w"]
    assert _fp16_ulps(ref.rmsnorm_ref(x, w, 1e-6), g[f"rms{i}_out"]).max() <= 1
    out, res = ref.rmsnorm_ref(x, w, 1e-6, residual=r)
    assert np.array_equal(_bits16(res), _bits16(g[f"rms{i}_res"]))  # fp16 add: bit-exact
    assert _fp16_ulps(out, g[f"rms{i}_out_res"]).max() <= 1


@pytest.mark.parametrize("i", range(4))
def test_swiglu_golden(golden, i):
    g = golden("norm_act")
    out = ref.swiglu_ref(g[f"swi{i}_g"], g[f"swi{i}_u"])
    assert _fp16_ulps(out, g[f"swi{i}_out"]).max() <= 1


def test_swiglu_edge_golden(golden):
    g = golden("norm_act")
    out = ref.swiglu_ref(g["swiedge_g"], g["swiedge_u"])
    assert _fp16_ulps(out, g["swiedge_out"]).max() <= 1


@pytest.mark.parametrize("case", ["fp80", "fp81", "fp82", "fp8edge"])
def test_fp8_quantize_bit_exact(golden, case):
    g = golden("fp8")
    wq, s = oracle.quantize_fp8(g[f"{case}_w"])
    assert np.array_equal(wq, g[f"{case}_wq"])
    assert np.array_equal(_bits16(s), _bits16(g[f"{case}_scale"]))
    deq = oracle.dequantize_fp8(g[f"{case}_wq"], g[f"{case}_scale"])
    assert np.array_equal(_bits16(deq), _bits16(g[f"{case}_deq"]))


def test_w8a16_golden(golden):
    g = golden("fp8")
    out = ref.w8a16_ref(g["w8_x"], g["w8_wq"], g["w8_scale"], g["w8_bias"])
    np.testing.assert_allclose(out, g["w8_ref"], rtol=1e-5, atol=1e-5)


def test_e4m3_roundtrip_all_codes():
    """Every finite e4m3fn code decodes and re-encodes to itself (format definition)."""
    lib = oracle.lib()
    import ctypes

    lib.oracle_e4m3_to_f32.restype = ctypes.c_float
    lib.oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
    lib.oracle_f32_to_e4m3.restype = ctypes.c_uint8
    lib.oracle_f32_to_e4m3.argtypes = [ctypes.c_float]
    for b in range(256):
        if b & 0x7F == 0x7F:
            continue
        v = lib.oracle_e4m3_to_f32(b)
        assert lib.oracle_f32_to_e4m3(v) == (b if v != 0 or b == 0 else b), b


def test_torch_cpu_restatement_golden(golden):
    """oracle.torch_ref (the reference's CPU W4A16 path on torch, used to time the CPU baseline)
    gives the reference's dequantized weights bit for bit, its unpacking matches the golden
    pack/unpack vectors, and its matmul matches the reference outputs."""
    import torch

    from oracle import torch_ref

    q = golden("quant")
    unpacked = torch_ref.unpack_int4(torch.from_numpy(q["pack_packed"]))
    assert np.array_equal(unpacked.numpy(), q["pack_unpacked"])
    g = golden("matmul")
    for i, (M, N, K, has_bias) in enumerate(g["w4_cases"]):
        x, qw, s, z = (torch.from_numpy(g[f"w4_{i}_{k}"]) for k in ("x", "qweight", "scales", "zeros"))
        if f"w4_{i}_deq" in g:
            deq = torch_ref.dequantize(qw, s, z, 128).contiguous().numpy()
            assert np.array_equal(_bits16(deq), _bits16(g[f"w4_{i}_deq"]))
        bias = torch.from_numpy(g[f"w4_{i}_bias"]) if has_bias else None
        out = torch_ref.w4a16_ref(x, qw, s, z, 128, bias).numpy()
        np.testing.assert_allclose(out, g[f"w4_{i}_ref"], rtol=1e-5, atol=1e-5)


def test_torch_quantize_rtn_golden(golden):
    """oracle.torch_ref.quantize_rtn reproduces the reference's golden quantizations bit for bit."""
    import torch

    from oracle import torch_ref

    g = golden("quant")
    for case in ("rtn0", "rtn1", "rtn2", "rtn3", "rtn4", "rtnedge"):
        qw, s, z = torch_ref.quantize_rtn(torch.from_numpy(g[f"{case}_w"]), 128)
        assert np.array_equal(qw.numpy(), g[f"{case}_qweight"]), case
        assert np.array_equal(_bits16(s.numpy()), _bits16(g[f"{case}_scales"])), case
        assert np.array_equal(_bits16(z.numpy()), _bits16(g[f"{case}_zeros"])), case


def _weights_strategy():
    from hypothesis import strategies as st
    from hypothesis.extra import numpy as hnp

    finite16 = st.floats(min_value=-60000, max_value=60000, allow_nan=False, allow_infinity=False, width=16)
    specials = st.sampled_from([0.0, -0.0, 1.0, -1.0, 6e-8, -6e-8, 1e-4, 65504.0, -65504.0, 0.5, 0.25])
    return st.tuples(st.integers(1, 4), st.sampled_from([128, 256])).flatmap(
        lambda nk: hnp.arrays(np.float16, (nk[0], nk[1]), elements=st.one_of(finite16, specials)))


def test_two_restatements_of_rtn_agree():
    """Property check of the quantizer's edge handling: the C restatement (oracle.quantize_rtn) and the
    torch one (oracle.torch_ref) agree on arbitrary fp16 groups - constants, signed zeros, subnormals,
    the fp16 extremes, mixed magnitudes: packed weights and scales bit for bit, zero points by value.
    A group whose minimum is a zero present with both signs is the one place the zero point's sign
    bit can differ: torch's min/max reductions return whichever signed zero their lane order keeps
    (a [+0, -0, ...] group gives -0, a [-0, +0, ...] one +0), the C loop the first one. The sign of a
    zero point changes no packed value and no dequantized weight ((q - (+0)) and (q - (-0)) are equal),
    and the defined cases (all +0, all -0) are pinned bit for bit by the golden vectors."""
    import torch
    from hypothesis import given, settings

    from oracle import torch_ref

    @settings(max_examples=300, deadline=None)
    @given(_weights_strategy())
    def check(w):
        qc, sc, zc = oracle.quantize_rtn(w, 128)
        qt, st_, zt = torch_ref.quantize_rtn(torch.from_numpy(w), 128)
        assert np.array_equal(qc, qt.numpy())
        assert np.array_equal(_bits16(sc), _bits16(st_.numpy()))
        assert np.array_equal(zc.astype(np.float32), zt.numpy().astype(np.float32))
        deq_c = oracle.dequantize_int4(qc, sc, zc, 128)
        deq_t = torch_ref.dequantize(qt, st_, zt, 128).contiguous().numpy()
        assert np.array_equal(deq_c.astype(np.float32), deq_t.astype(np.float32))

    check()


def test_two_restatements_of_fp8_agree():
    """The C e4m3 quantizer (oracle.quantize_fp8, its own round-to-nearest-even encoder) and torch's
    float8_e4m3fn cast as the reference uses it (oracle.torch_ref.quantize_fp8) agree bit for bit on
    arbitrary fp16 rows: zeros, subnormals, fp16 extremes, values that land on e4m3 rounding ties."""
    import torch
    from hypothesis import given, settings

    from oracle import torch_ref

    @settings(max_examples=300, deadline=None)
    @given(_weights_strategy())
    def check(w):
        qc, sc = oracle.quantize_fp8(w)
        qt, st_ = torch_ref.quantize_fp8(torch.from_numpy(w))
        assert np.array_equal(_bits16(sc), _bits16(st_.numpy()))
        assert np.array_equal(qc, qt.numpy())

    check()


def _ulps_f16(a, b):
    a = _bits16(np.asarray(a, dtype=np.float16)).astype(np.int32)
    b = _bits16(np.asarray(b, dtype=np.float16)).astype(np.int32)
    a = np.where(a & 0x8000, 0x8000 - a, a)
    b = np.where(b & 0x8000, 0x8000 - b, b)
    return np.abs(a - b)


def test_rmsnorm_and_swiglu_restatements_agree():
    """The numpy oracle's RMSNorm and SwiGLU against the reference's torch formulation on random rows
    (hypothesis): residual outputs bit for bit, normalized outputs and activations within one fp16 ulp
    (numpy and torch may round rsqrt / exp in fp32 differently by an ulp before the fp16 rounding)."""
    import torch
    from hypothesis import given, settings
    from hypothesis import strategies as st
    from hypothesis.extra import numpy as hnp

    from oracle import torch_ref

    vals = st.floats(min_value=-8, max_value=8, allow_nan=False, width=16)

    @settings(max_examples=150, deadline=None)
    @given(st.integers(1, 3).flatmap(lambda m: st.tuples(
        hnp.arrays(np.float16, (m, 64), elements=vals), hnp.arrays(np.float16, (m, 64), elements=vals),
        hnp.arrays(np.float16, (64,), elements=st.floats(0.5, 1.5, width=16)))))
    def check(args):
        x, r, w = args
        out_n, res_n = ref.rmsnorm_ref(x, w, 1e-6, residual=r)
        out_t, res_t = torch_ref.rmsnorm_ref(torch.from_numpy(x), torch.from_numpy(w), 1e-6, torch.from_numpy(r))
        assert np.array_equal(_bits16(res_n), _bits16(res_t.numpy()))
        assert (_ulps_f16(out_n, out_t.numpy()) <= 1).all()
        act_n = ref.swiglu_ref(x, r)
        act_t = torch_ref.swiglu_ref(torch.from_numpy(x), torch.from_numpy(r))
        assert (_ulps_f16(act_n, act_t.numpy()) <= 1).all()

    check()
