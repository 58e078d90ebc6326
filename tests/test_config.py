"""The `config=` dict of w4a16_matmul / w8a16_matmul and the per-shape choice helpers (CPU only).

The reference passes Triton-style dicts (tests/test_w4a16.py:33,51 of the reference); here SPLIT_K
maps to the cluster split-K factor, BLOCK_N to the CTA column tile, and the extra keys to flags of
dk_matmul_config. export_choices / import_choices keep the reference's key format
(kernels/w4a16.py:333-342 of the reference)."""

import pytest

from kernels import _lib
from kernels.w4a16 import _config, export_choices, import_choices


def test_empty_config_is_automatic():
    for cfg in (None, {}):
        c = _config(cfg)
        assert (c.split_k, c.block_n, c.flags, c.n_prefetch) == (0, 0, 0, 0)


def test_reference_triton_dicts():
    c = _config(dict(BLOCK_M=16, BLOCK_N=32, BLOCK_K=64, SPLIT_K=1, GROUP_M=8))
    assert (c.split_k, c.block_n, c.flags) == (1, 32, 0)
    c = _config(dict(GEMV=True, BLOCK_N=128, BLOCK_K=64, SPLIT_K=3))
    assert (c.split_k, c.block_n) == (3, 128)


@pytest.mark.parametrize("bn,want", [(32, 32), (64, 64), (128, 128), (256, 256), (48, 0), (512, 0), (None, 0)])
def test_block_n_values(bn, want):
    assert _config({"BLOCK_N": bn}).block_n == want


def test_split_k_limits():
    assert _config({"SPLIT_K": 8}).split_k == 8
    assert _config({"SPLIT_K": 0}).split_k == 0
    assert _config({"SPLIT_K": -2}).split_k == 0
    with pytest.raises(RuntimeError, match="cluster limit"):
        _config({"SPLIT_K": 9})


def test_flags():
    assert _config({"STATIC_WEIGHTS": True}).flags == _lib.FLAG_STATIC_WEIGHTS
    assert _config({"GENERIC": True}).flags == _lib.FLAG_GENERIC
    assert _config({"EXACT": True}).flags == _lib.FLAG_EXACT_DEQUANT
    assert _config({"FACTORED": False}).flags == _lib.FLAG_EXACT_DEQUANT  # the reference's unfactored numerics
    assert _config({"FACTORED": True}).flags == 0
    assert _config({"DECODE_GEMV": True}).flags == _lib.FLAG_GEMV
    both = _config({"STATIC_WEIGHTS": True, "DECODE_GEMV": True}).flags
    assert both == _lib.FLAG_STATIC_WEIGHTS | _lib.FLAG_GEMV


def test_choices_roundtrip():
    before = export_choices()
    import_choices({"1,2048,1536,False": {"SPLIT_K": "auto", "BLOCK_N": "auto"},
                    "16,17920,1536,True": {"SPLIT_K": 2, "BLOCK_N": 64}})
    got = export_choices()
    assert got["1,2048,1536,False"] == {"SPLIT_K": "auto", "BLOCK_N": "auto"}
    assert got["16,17920,1536,True"] == {"SPLIT_K": 2, "BLOCK_N": 64}
    assert set(before) <= set(got)
