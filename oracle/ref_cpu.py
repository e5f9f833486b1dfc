"""Run the reference's compiled CPU libraries from oracle/_ref (TEST
INFRASTRUCTURE ONLY: parity pin of the oracle and the CPU baseline of bench.py).

The libraries export the reference ABI ``void run_einsum(const float*,
const float*, float*, void*)`` (templates.py:151-155); the reference runner
feeds operands swapped when its planner chose the swapped order
(builder.py:853-854), which the manifest records.
"""
import ctypes
import json
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
_libs = {}
_lock = threading.Lock()


def available() -> bool:
    return os.path.exists(os.path.join(REF_DIR, "manifest.json"))


def _manifest():
    with open(os.path.join(REF_DIR, "manifest.json")) as f:
        return json.load(f)


def names():
    return sorted(_manifest())


def spec(name):
    return _manifest()[name]


def _lib(name):
    with _lock:
        if name not in _libs:
            L = ctypes.CDLL(os.path.join(REF_DIR, f"{name}.so"))
            L.run_einsum.argtypes = [ctypes.c_void_p] * 4
            L.run_einsum.restype = None
            _libs[name] = L
        return _libs[name]


def sample_inputs(name, seed=0):
    s = spec(name)
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(s["shape0"], dtype=np.float32),
            rng.standard_normal(s["shape1"], dtype=np.float32))


def run(name, a, b, out=None):
    """One call of the reference CPU library `name` on fp32 arrays."""
    s = spec(name)
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    if out is None:
        out = np.zeros(s["out_shape"], dtype=np.float32)
    x, y = (b, a) if s["swap"] else (a, b)
    _lib(name).run_einsum(ctypes.c_void_p(x.ctypes.data), ctypes.c_void_p(y.ctypes.data),
                          ctypes.c_void_p(out.ctypes.data), None)
    return out
