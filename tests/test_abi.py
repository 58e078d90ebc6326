"""The C-ABI library builds for sm_100a, loads, and exports every entry point its header declares
(no GPU needed: nothing is called that touches a device)."""

import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "decodek.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(dk_\w+)\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("dk_w4a16_matmul", "dk_quantize_rtn", "dk_pack_int4", "dk_rmsnorm", "dk_swiglu"):
        assert name in syms


def test_library_builds_and_exports_every_symbol():
    import importlib.util

    spec = importlib.util.spec_from_file_location("dk_build", ROOT / "llm-decode-kernels_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    lib = mod.build()
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (dk_\w+)", out.stdout))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_library_loads_and_reports_version():
    from kernels import _lib

    h = _lib.lib()
    assert h.dk_abi_version() == 6
    for name in declared_symbols():
        assert hasattr(h, name)
    # every declared symbol has a ctypes signature in the Python mirror
    missing = [s for s in declared_symbols() if s not in _lib.SIGNATURES and s != "dk_last_error"]
    assert not missing, missing


def test_errors_come_back_as_status_without_a_gpu():
    """Argument checks run before any CUDA call, so they work on a machine without a GPU."""
    import ctypes

    from kernels import _lib

    h = _lib.lib()
    rc = h.dk_w4a16_matmul(None, 100, None, None, None, None, None, 100, 1, 8, 100, 128, None, None)
    assert rc == -1 and b"group_size" in h.dk_last_error()
    rc = h.dk_pack_int4(None, None, 12, 4, None)
    assert rc == -1 and b"multiple of 8" in h.dk_last_error()
    cfg = _lib.MatmulConfig()
    assert ctypes.sizeof(cfg) == h.dk_matmul_config_size() == 16 + 16 * _lib.MAX_L2_PREFETCH


def test_package_has_no_oracle_or_cpu_path():
    """The product package never imports the oracle and has no torch-CPU fallback."""
    pkg = ROOT / "llm-decode-kernels_b200" / "kernels"
    for py in pkg.rglob("*.py"):
        text = py.read_text()
        assert "import oracle" not in text and "from oracle" not in text, py


def test_tp_entry_points_validate_without_a_gpu():
    """The tensor-parallel set-up calls check their arguments before touching the device."""
    import ctypes

    from kernels import _lib

    h = _lib.lib()
    n = ctypes.c_uint64(0)
    assert h.dk_tp_buffer_bytes(2, 16, 3584, ctypes.byref(n)) == 0
    assert n.value == 256 + 2 * 2 * 16 * 3584 * 8
    assert h.dk_tp_buffer_bytes(9, 16, 3584, ctypes.byref(n)) == -1
    assert h.dk_tp_buffer_bytes(2, 64, 3584, ctypes.byref(n)) == 0  # up to 64 rows (the small-M kernel)
    assert h.dk_tp_buffer_bytes(2, 65, 3584, ctypes.byref(n)) == -1
    assert h.dk_tp_buffer_bytes(2, 16, 3585, ctypes.byref(n)) == -1
    comm = ctypes.c_void_p()
    bufs = (ctypes.c_void_p * 2)(None, None)
    assert h.dk_tp_comm_create(ctypes.byref(comm), 0, 2, bufs, 16, 3584) == -1
    assert b"NULL" in h.dk_last_error()
    rc = h.dk_w4a16_matmul_allreduce(None, 128, None, None, None, None, None, 8, 1, 8, 128, 128, None, None, None)
    assert rc == -1
