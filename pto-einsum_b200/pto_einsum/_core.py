"""Locate, build and load the sm_100a core library ``libpto_einsum_b200.so``.

The core library is compiled in-tree (``pto_einsum/_lib``) from ``csrc/`` with
nvcc for ``sm_100a``. There is no CPU or Python fallback: if the library is
missing and cannot be built, every device entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libpto_einsum_b200.so")
CSRC_DIR = os.path.join(os.path.dirname(PKG_DIR), "csrc")
# Headers: repo-level include/ (source checkout) or a packaged copy.
_CANDIDATE_INCLUDES = [
    os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include"),
    os.path.join(PKG_DIR, "include"),
]
INCLUDE_DIR = next((p for p in _CANDIDATE_INCLUDES if os.path.exists(os.path.join(p, "pto_einsum_b200.h"))),
                   _CANDIDATE_INCLUDES[0])

_lock = threading.Lock()
_lib = None

PE_F32, PE_F16 = 0, 1


def build_core(force: bool = False) -> str:
    """Compile the core library with nvcc (sm_100a) if it is missing or stale."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_pe_csrc_build", os.path.join(CSRC_DIR, "build.py"))
    if spec is None or not os.path.exists(os.path.join(CSRC_DIR, "build.py")):
        raise RuntimeError(f"pto_einsum: CUDA sources not found under {CSRC_DIR}; cannot build "
                           f"{LIB_PATH}")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(force=force)


def _declare(lib):
    c = ctypes
    lib.pe_last_error.restype = c.c_int
    lib.pe_error_string.restype = c.c_char_p
    lib.pe_error_string.argtypes = [c.c_int]
    lib.pe_device_error.restype = c.c_int
    lib.pe_device_error.argtypes = [c.c_void_p]
    lib.pe_launch_count.restype = c.c_int64
    lib.pe_selftest_wait_timeout.argtypes = [c.c_uint64, c.c_void_p]
    lib.pe_selftest_wait_timeout.restype = c.c_int
    lib.pe_version.restype = c.c_char_p
    lib.pe_stream_synchronize.argtypes = [c.c_void_p]
    lib.pe_elementwise_mul.argtypes = [c.c_int32, c.c_void_p, c.c_void_p, c.c_void_p, c.c_int64, c.c_void_p]
    lib.pe_batched_matmul.argtypes = [c.c_int32, c.c_int64, c.c_int64, c.c_int64, c.c_int64,
                                      c.c_void_p, c.c_void_p, c.c_void_p, c.c_void_p]
    return lib


def core_lib():
    """Load (building first if needed) and return the core library handle."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        stale = not os.path.exists(LIB_PATH)
        if not stale and os.path.isdir(CSRC_DIR):
            try:
                import importlib.util
                spec = importlib.util.spec_from_file_location(
                    "_pe_csrc_build", os.path.join(CSRC_DIR, "build.py"))
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                stale = mod.needs_build()
            except Exception:
                stale = False
        if stale:
            build_core()
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"pto_einsum: CUDA core library missing: {LIB_PATH}")
        _lib = _declare(ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL))
        return _lib


def core_version() -> str:
    return core_lib().pe_version().decode()


def error_string(code: int) -> str:
    return core_lib().pe_error_string(int(code)).decode()


def launch_count() -> int:
    """Number of core kernels launched by this process so far."""
    return int(core_lib().pe_launch_count())


def device_error(stream_ptr: int = 0) -> int:
    """Synchronise the stream and return (and clear) the device error word."""
    return int(core_lib().pe_device_error(ctypes.c_void_p(stream_ptr)))
