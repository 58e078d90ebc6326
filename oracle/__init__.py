"""CPU oracle for the decode hot path. TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py` may import this
package, and only as the checker (or the timed CPU baseline). The product path in
`llm-decode-kernels_b200/kernels` never imports it and has no CPU fallback.

Contents (each function cites the reference file:line it restates):
- `quant_ref.c` (built into `liboracle.so` by `build()`): bit-exact pack/unpack, RTN int4
  quantization and e4m3 quantization.
- `ref.py`: numpy restatements of the float references (`kernels/reference.py`,
  `kernels/fp8.py`) and a torch-CPU restatement of the Qwen2 decode runner.

Pinning: every function here is checked against golden vectors produced by the reference's own
code (`tests/golden/make_golden.py`) in `tests/test_oracle.py`.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


def build(force: bool = False) -> Path:
    """Compile quant_ref.c with IEEE fp32 semantics (no FMA contraction, no fast-math)."""
    src = HERE / "quant_ref.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
        subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math",
                        "-fPIC", "-shared", str(src), "-o", str(tmp), "-lm"], check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        P, I = ctypes.c_void_p, ctypes.c_int64
        for name, args in {
            "oracle_pack_int4": [P, I, I, P],
            "oracle_unpack_int4": [P, I, I, P],
            "oracle_quantize_rtn": [P, I, I, I, P, P, P],
            "oracle_dequantize_int4": [P, P, P, I, I, I, P],
            "oracle_quantize_fp8": [P, I, I, P, P],
            "oracle_dequantize_fp8": [P, P, I, I, P],
        }.items():
            getattr(_lib, name).argtypes = args
            getattr(_lib, name).restype = None
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def pack_int4(q: np.ndarray) -> np.ndarray:
    """[K, N] ints -> [K/8, N] int32 (kernels/quant.py:20-28)."""
    q = np.ascontiguousarray(q, dtype=np.int32)
    K, N = q.shape
    assert K % 8 == 0, "K must be a multiple of 8"
    out = np.empty((K // 8, N), dtype=np.int32)
    lib().oracle_pack_int4(_p(q), K, N, _p(out))
    return out


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """[K/8, N] int32 -> [K, N] int32 in 0..15 (kernels/quant.py:31-35)."""
    packed = np.ascontiguousarray(packed, dtype=np.int32)
    R, N = packed.shape
    out = np.empty((R * 8, N), dtype=np.int32)
    lib().oracle_unpack_int4(_p(packed), R * 8, N, _p(out))
    return out


def quantize_rtn(w: np.ndarray, group_size: int = 128):
    """fp16 [N, K] -> (qweight int32 [K/8, N], scales fp16 [K/G, N], zeros fp16 [K/G, N])
    (kernels/quant.py:38-49)."""
    w = np.ascontiguousarray(w, dtype=np.float16)
    N, K = w.shape
    assert K % group_size == 0 and group_size % 8 == 0
    qw = np.empty((K // 8, N), dtype=np.int32)
    s = np.empty((K // group_size, N), dtype=np.float16)
    z = np.empty((K // group_size, N), dtype=np.float16)
    lib().oracle_quantize_rtn(_p(w), N, K, group_size, _p(qw), _p(s), _p(z))
    return qw, s, z


def dequantize_int4(qweight, scales, zeros, group_size: int = 128) -> np.ndarray:
    """-> fp16 [N, K] (kernels/reference.py:27-36)."""
    qweight = np.ascontiguousarray(qweight, dtype=np.int32)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    zeros = np.ascontiguousarray(zeros, dtype=np.float16)
    K, N = qweight.shape[0] * 8, qweight.shape[1]
    out = np.empty((N, K), dtype=np.float16)
    lib().oracle_dequantize_int4(_p(qweight), _p(scales), _p(zeros), N, K, group_size, _p(out))
    return out


def quantize_fp8(w: np.ndarray):
    """fp16 [N, K] -> (e4m3 bytes uint8 [K, N], scale fp16 [N]) (kernels/fp8.py:25-30)."""
    w = np.ascontiguousarray(w, dtype=np.float16)
    N, K = w.shape
    wq = np.empty((K, N), dtype=np.uint8)
    s = np.empty((N,), dtype=np.float16)
    lib().oracle_quantize_fp8(_p(w), N, K, _p(wq), _p(s))
    return wq, s


def dequantize_fp8(wq: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """e4m3 bytes [K, N] + fp16 [N] -> fp16 [N, K] (kernels/fp8.py:33-35)."""
    wq = np.ascontiguousarray(wq, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.float16)
    K, N = wq.shape
    out = np.empty((N, K), dtype=np.float16)
    lib().oracle_dequantize_fp8(_p(wq), _p(scale), N, K, _p(out))
    return out


def weight_bytes(N: int, K: int, group_size: int = 128) -> int:
    """Packed int4 bytes + fp16 scales and zeros (kernels/quant.py:52-54)."""
    return N * K // 2 + 2 * (K // group_size) * N * 2
