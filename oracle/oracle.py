"""CPU parity oracle - TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arms may import this module; the product package (pto_einsum) never does.

It restates the reference's CPU path:
  * planning of the transpose -> batched matmul -> transpose recipe with
    ``device="cpu"`` semantics (src/pto_einsum/builder.py:148-367; on CPU the
    broadcast classifier is skipped, builder.py:373-376, so broadcast
    equations take the matmul route with C = 1),
  * execution through einsum_oracle.c (restating include/cpu_einsum.h),
  * fp16 inputs are upcast to fp32 first: the reference CPU kernel casts every
    operand with static_cast<float> before multiplying (cpu_einsum.h:75, :90),
    so the upcast is exact and changes nothing.

Parity pin: tests/test_oracle.py checks this oracle against the golden outputs
in tests/golden/, which were produced by running the reference's own CPU path
(tests/golden/make_golden.py), and, when oracle/_ref is built, against the
reference libraries directly.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from math import prod

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD_DIR, "libeinsum_oracle.so")
SRC = os.path.join(HERE, "einsum_oracle.c")

_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> str:
    """Compile einsum_oracle.c with gcc (no FMA contraction)."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(BUILD_DIR, exist_ok=True)
    tmp = f"{LIB}.{os.getpid()}.tmp"
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC", "-pthread",
           SRC, "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stderr)
    os.replace(tmp, LIB)
    return LIB


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(LIB)
            P = ctypes.c_void_p
            i64 = ctypes.c_int64
            L.oracle_einsum_f32.argtypes = [P, P, P, ctypes.c_int, P, P, ctypes.c_int, P, P, ctypes.c_int, P, P,
                                            i64, i64, i64, i64, ctypes.c_int]
            L.oracle_batched_matmul_f32.argtypes = [P, P, P, i64, i64, i64, i64, ctypes.c_int]
            L.oracle_transpose_f32.argtypes = [P, P, ctypes.c_int, P, P]
            L.oracle_elementwise_f32.argtypes = [P, P, P, i64]
            L.oracle_broadcast_f32.argtypes = [P, P, P, ctypes.c_int, i64, i64, i64, ctypes.c_int, P, P]
            _lib = L
        return _lib


# ---------------------------------------------------------------------------
# planning with device="cpu" semantics (builder.py:148-367)
# ---------------------------------------------------------------------------

def _split(eq: str):
    lhs, out = (s.strip() for s in eq.split('->'))
    a, b = (s.strip() for s in lhs.split(','))
    return a, b, out


def _strides(shape):
    st, run = [0] * len(shape), 1
    for p in reversed(range(len(shape))):
        st[p] = run
        run *= int(shape[p])
    return st


def cpu_plan(eq: str, shape0, shape1) -> dict:
    """Transpose configs + matmul sizes of the reference CPU path.

    Returns None-free dict with keys: elementwise, perm0, perm1, out_interp,
    out_perm, I, L0, L1, C, out_shape.
    """
    a, b, o = _split(eq)
    size = {}
    for ch, d in zip(b, shape1):
        size[ch] = int(d)
    for ch, d in zip(a, shape0):
        size[ch] = int(d)
    out_shape = tuple(size[ch] for ch in o)
    if list(a) == list(b) == list(o):
        return dict(elementwise=True, out_shape=out_shape, n=prod(out_shape))
    sa, sb, so = set(a), set(b), set(o)
    common = sa & sb
    contract = sorted(common - so, key=b.index)
    batch = sorted(common & so, key=b.index)
    free0 = sorted((so - common) & sa, key=a.index)
    free1 = sorted((so - common) & sb, key=b.index)
    solo = (sa - sb - so) | (sb - sa - so)
    if solo:
        raise ValueError(f"single-operand reduction ({sorted(solo)}) is not supported")
    perm0 = tuple(a.index(c) for c in batch + free0 + contract)
    perm1 = tuple(b.index(c) for c in batch + contract + free1)
    interp = batch + free0 + free1
    out_perm = tuple(sorted(range(len(interp)), key=lambda j: o.index(interp[j])))
    return dict(elementwise=False, perm0=perm0, perm1=perm1,
                out_interp=tuple(size[c] for c in interp), out_perm=out_perm,
                I=prod(size[c] for c in batch), L0=prod(size[c] for c in free0),
                L1=prod(size[c] for c in free1), C=prod(size[c] for c in contract),
                out_shape=out_shape)


def _tcfg(shape, perm):
    st = _strides(shape)
    to = np.array([shape[p] for p in perm], dtype=np.int64)
    ps = np.array([st[p] for p in perm], dtype=np.int64)
    return len(shape), to, ps


def _as_f32(x) -> np.ndarray:
    try:
        import torch
        if isinstance(x, torch.Tensor):
            x = x.detach().cpu().float().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def einsum_cpu(eq: str, x, y, threads: int = 1) -> np.ndarray:
    """Reference CPU einsum of two operands; returns fp32 ndarray."""
    a, b = _as_f32(x), _as_f32(y)
    plan = cpu_plan(eq, a.shape, b.shape)
    out = np.zeros(plan['out_shape'], dtype=np.float32)
    if out.size == 0:
        return out
    L = lib()
    if plan['elementwise']:
        L.oracle_elementwise_f32(_p(a), _p(b), _p(out), out.size)
        return out
    d0, to0, ps0 = _tcfg(a.shape, plan['perm0'])
    d1, to1, ps1 = _tcfg(b.shape, plan['perm1'])
    do, too, pso = _tcfg(plan['out_interp'], plan['out_perm'])
    rc = L.oracle_einsum_f32(_p(a), _p(b), _p(out), d0, _p(to0), _p(ps0), d1, _p(to1), _p(ps1),
                             do, _p(too), _p(pso), plan['I'], plan['L0'], plan['L1'], plan['C'], threads)
    if rc:
        raise MemoryError("oracle_einsum_f32 could not allocate its buffers")
    return out


def batched_matmul_cpu(a, b, threads: int = 1) -> np.ndarray:
    """o[I,L0,L1] = a[I,L0,C] x b[I,C,L1] in the reference accumulation order."""
    a, b = _as_f32(a), _as_f32(b)
    I, L0, C = a.shape
    L1 = b.shape[2]
    out = np.zeros((I, L0, L1), dtype=np.float32)
    lib().oracle_batched_matmul_f32(_p(a), _p(b), _p(out), I, L0, L1, C, threads)
    return out


def transpose_cpu(x, perm) -> np.ndarray:
    a = _as_f32(x)
    d, to, ps = _tcfg(a.shape, perm)
    out = np.zeros(tuple(int(t) for t in to), dtype=np.float32)
    lib().oracle_transpose_f32(_p(a), _p(out), d, _p(to), _p(ps))
    return out


def broadcast_cpu(recipe: dict, x, y) -> np.ndarray:
    """Broadcast route (recipe from the CUDA planner) evaluated on the CPU."""
    a, b = _as_f32(x), _as_f32(y)
    full, bc = (a, b) if recipe['bc_full_is_in0'] else (b, a)
    out = np.zeros(recipe['out_shape'], dtype=np.float32)
    dims = np.array(recipe['bc_outer_dims'] or (1,), dtype=np.int64)
    bst = np.array(recipe['bc_outer_bstride'] or (0,), dtype=np.int64)
    lib().oracle_broadcast_f32(_p(full), _p(bc), _p(out), recipe['bc_mode'], out.size, recipe['bc_Cc'],
                               recipe['bc_Inner'], len(recipe['bc_outer_dims']), _p(dims), _p(bst))
    return out


def rel_frobenius(x, ref) -> float:
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref.ravel())
    num = np.linalg.norm((x - ref).ravel())
    return float(num / den) if den > 0 else float(num)
