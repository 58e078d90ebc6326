"""Loader for `libdecodek.so`, the C ABI of the sm_100a kernels (declared in include/decodek.h).

Every op in this package calls the library through ctypes with raw device pointers and torch's
current CUDA stream. There is no CPU fallback: a CPU tensor, a missing library or a non-B200 device
raises. A negative status from the library becomes a RuntimeError carrying `dk_last_error()`.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parents[1] / "lib" / "libdecodek.so"

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int32
F32 = ctypes.c_float


MAX_L2_PREFETCH = 6


class MatmulConfig(ctypes.Structure):
    """dk_matmul_config: zero fields mean "choose automatically"; n_prefetch ranges of device memory
    the launch pulls into L2 for a later launch."""

    _fields_ = [("split_k", I32), ("block_n", I32), ("flags", I32), ("n_prefetch", I32),
                ("l2_prefetch_ptr", ctypes.c_void_p * MAX_L2_PREFETCH),
                ("l2_prefetch_bytes", ctypes.c_uint64 * MAX_L2_PREFETCH)]


class StepLayer(ctypes.Structure):
    """dk_step_layer: one decoder layer's tensors for the fused decode step (device pointers)."""

    _fields_ = [(name, P) for name in (
        "input_norm", "post_norm",
        "qkv_qweight", "qkv_scales", "qkv_zeros", "qkv_bias",
        "o_qweight", "o_scales", "o_zeros", "o_bias",
        "gate_up_qweight", "gate_up_scales", "gate_up_zeros", "gate_up_bias",
        "down_qweight", "down_scales", "down_zeros", "down_bias")]


class StepModel(ctypes.Structure):
    """dk_step_model: sizes and tensors of the model the fused decode step runs."""

    _fields_ = [("n_layers", I32), ("hidden", I32), ("n_heads", I32), ("n_kv", I32), ("head_dim", I32),
                ("intermediate", I32), ("vocab", I32), ("max_len", I32), ("batch", I32), ("eps", F32),
                ("embed", P), ("final_norm", P), ("lm_head", P), ("rope_cos", P), ("rope_sin", P),
                ("k_cache", P), ("v_cache", P), ("layers", ctypes.POINTER(StepLayer))]


FLAG_STATIC_WEIGHTS = 1
FLAG_GENERIC = 2
FLAG_EXACT_DEQUANT = 4
FLAG_GEMV = 8

# name -> argtypes; every function returns int status
SIGNATURES = {
    "dk_abi_version": [],
    "dk_matmul_config_size": [],
    "dk_device_error": [ctypes.POINTER(I32)],
    "dk_clear_device_error": [],
    "dk_set_pdl": [I32],
    "dk_pack_int4": [P, P, I64, I64, P],
    "dk_unpack_int4": [P, P, I64, I64, P],
    "dk_quantize_rtn": [P, I64, P, P, P, I64, I64, I64, P],
    "dk_dequantize_int4": [P, P, P, P, I64, I64, I64, P],
    "dk_w4a16_matmul": [P, I64, P, P, P, P, P, I64, I64, I64, I64, I64, ctypes.POINTER(MatmulConfig), P],
    "dk_w4a16_swiglu": [P, I64, P, P, P, P, P, I64, I64, I64, I64, I64, ctypes.POINTER(MatmulConfig), P],
    "dk_w4a16_rmsnorm_matmul": [P, I64, P, I64, P, F32, P, I64, P, P, P, P, P, I64, I64, I64, I64, I64, I32,
                                ctypes.POINTER(MatmulConfig), P],
    "dk_w4a16_matmul_partials": [P, I64, P, P, P, I64, I64, I64, I64, P, I64, ctypes.POINTER(I32),
                                 ctypes.POINTER(MatmulConfig), P],
    "dk_w4a16_rmsnorm_matmul_partials": [P, I32, P, P, I64, P, F32, P, I64, P, P, P, P, P, I64, I64, I64, I64, I64,
                                         I32, ctypes.POINTER(MatmulConfig), P],
    "dk_quantize_fp8": [P, I64, P, P, I64, I64, P],
    "dk_dequantize_fp8": [P, P, P, I64, I64, P],
    "dk_w8a16_matmul": [P, I64, P, P, P, P, I64, I64, I64, I64, ctypes.POINTER(MatmulConfig), P],
    "dk_rmsnorm": [P, I64, P, I64, P, P, I64, P, I64, I64, I64, F32, P],
    "dk_swiglu": [P, I64, P, I64, P, I64, I64, I64, P],
    "dk_decode_attention": [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I32, I32, P],
    "dk_lm_head_greedy_workspace_bytes": [ctypes.POINTER(ctypes.c_uint64)],
    "dk_lm_head_greedy": [P, P, P, F32, P, I64, I64, I64, P, P, P, I64, I64, P, P, ctypes.c_uint64, P],
    "dk_embed_tokens": [P, P, I64, I64, I64, P, P],
    "dk_tp_buffer_bytes": [I32, I64, I64, ctypes.POINTER(ctypes.c_uint64)],
    "dk_tp_buffer_alloc": [ctypes.c_uint64, ctypes.POINTER(P), P],
    "dk_tp_buffer_free": [P],
    "dk_tp_buffer_open": [P, ctypes.POINTER(P)],
    "dk_tp_buffer_close": [P],
    "dk_tp_comm_create": [ctypes.POINTER(P), I32, I32, ctypes.POINTER(P), I64, I64],
    "dk_tp_comm_destroy": [P],
    "dk_tp_comm_set_wait": [P, ctypes.c_uint64],
    "dk_w4a16_matmul_allreduce": [P, I64, P, P, P, P, P, I64, I64, I64, I64, I64, ctypes.POINTER(MatmulConfig), P,
                                  P],
    "dk_w4a16_matmul_reduce_static": [P, I64, P, P, P, P, P, I64, I64, I64, I64, I64, ctypes.POINTER(MatmulConfig),
                                      P],
    "dk_step_workspace_bytes": [ctypes.POINTER(StepModel), ctypes.POINTER(ctypes.c_uint64)],
    "dk_step_create": [ctypes.POINTER(StepModel), P, ctypes.c_uint64, ctypes.POINTER(P)],
    "dk_step_run": [P, P, P, P, I64, P, P],
    "dk_step_destroy": [P],
    "dk_step_trace_bytes": [P, ctypes.POINTER(ctypes.c_uint64)],
    "dk_step_trace": [P, P, P, P, I64, P, P, P],
    "dk_step_ops": [P, ctypes.POINTER(I32), I32, ctypes.POINTER(I32)],
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python llm-decode-kernels_b200/build.py` "
                        "(the decode kernels have no CPU fallback)")
                h = ctypes.CDLL(str(LIB_PATH))
                for name, args in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.argtypes = args
                    fn.restype = ctypes.c_int
                h.dk_last_error.argtypes = []
                h.dk_last_error.restype = ctypes.c_char_p
                _lib = h
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().dk_last_error().decode(errors="replace")
        raise RuntimeError(f"{what}: {msg} (status {status})")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_extent(ok: bool, message: str) -> None:
    """Argument extents the kernels cannot see (they get raw pointers and sizes): a ValueError, raised
    whether or not Python runs with -O, so a short tensor is never read past its end."""
    if not ok:
        raise ValueError(message)


def reference_assert(ok: bool, message: str = "") -> None:
    """A check the reference makes with `assert` (same AssertionError), raised explicitly so that it
    also holds under python -O."""
    if not ok:
        raise AssertionError(message)


def require_cuda(what: str, *tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{what}: tensors must be on a CUDA device (no CPU path), got {t.device}")


def require_dtype(what: str, dtype: torch.dtype, *tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and t.dtype != dtype:
            raise RuntimeError(f"{what}: expected {dtype}, got {t.dtype}")


def device_error() -> int:
    """The library's device error word on the current device (0 = no bounded wait gave up)."""
    code = I32(0)
    call("dk_device_error", ctypes.byref(code))
    return code.value


def clear_device_error() -> None:
    call("dk_clear_device_error")


def set_pdl(enabled: bool) -> None:
    call("dk_set_pdl", int(bool(enabled)))
