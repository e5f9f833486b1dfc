"""pe_contract_noalloc: the contraction entry point that allocates nothing.

Callers that cannot allocate device memory at call time (fixed memory
budgets, foreign allocators, latency-critical paths) use pe_contract_noalloc,
whose scratch is a fixed array inside the library. These tests call it
through the C ABI and check it against the ordinary entry point (the
EinsumBuilder runner, which uses pe_contract with a cudaMalloc'd workspace),
twice in a row, because consecutive calls share and reuse the same array.
The file is named to be collected last.
"""
import ctypes

import pytest
import torch

from gpu_util import check_close, seeded
from oracle import oracle
from pto_einsum import EinsumBuilder, _core

pytestmark = pytest.mark.gpu

MAXR = 8


class ContractPlan(ctypes.Structure):
    """ctypes mirror of pe_contract_plan (include/pto_einsum_b200.h)."""
    _fields_ = [("dtype", ctypes.c_int32), ("rank0", ctypes.c_int32), ("rank1", ctypes.c_int32),
                ("out_rank", ctypes.c_int32),
                ("shape0", ctypes.c_int64 * MAXR), ("shape1", ctypes.c_int64 * MAXR),
                ("perm0", ctypes.c_int32 * MAXR), ("perm1", ctypes.c_int32 * MAXR),
                ("out_interp_shape", ctypes.c_int64 * MAXR), ("out_perm", ctypes.c_int32 * MAXR),
                ("n_batch", ctypes.c_int32), ("n_free0", ctypes.c_int32), ("n_free1", ctypes.c_int32),
                ("n_contract", ctypes.c_int32),
                ("I", ctypes.c_int64), ("L0", ctypes.c_int64), ("L1", ctypes.c_int64), ("C", ctypes.c_int64)]


def plan_of(builder):
    r = builder.recipe
    s0, s1 = builder._exec_shapes
    p = ContractPlan()
    p.dtype = 0 if builder.dtype == torch.float32 else 1
    p.rank0, p.rank1, p.out_rank = len(s0), len(s1), len(r["out_interpret_shape"])
    for k, d in enumerate(s0):
        p.shape0[k] = d
    for k, d in enumerate(s1):
        p.shape1[k] = d
    for k, q in enumerate(r["in_transpose_idxs"][0]):
        p.perm0[k] = q
    for k, q in enumerate(r["in_transpose_idxs"][1]):
        p.perm1[k] = q
    for k, d in enumerate(r["out_interpret_shape"]):
        p.out_interp_shape[k] = d
    for k, q in enumerate(r["out_transpose_idxs"]):
        p.out_perm[k] = q
    p.n_batch, p.n_free0, p.n_free1, p.n_contract = builder._axes
    p.I, p.L0, p.L1, p.C = r["I"], r["L0"], r["L1"], r["C"]
    return p


def lib():
    L = _core.core_lib()
    L.pe_contract_noalloc.argtypes = [ctypes.c_void_p] * 5
    L.pe_contract_noalloc.restype = ctypes.c_int
    L.pe_noalloc_scratch_bytes.restype = ctypes.c_size_t
    return L


class PoolUsage:
    """High-water mark of the device's default stream-ordered memory pool (the
    pool cudaMallocAsync draws from), read through the driver API: a call that
    allocated scratch, even if it freed it again, raises the mark."""
    USED_MEM_CURRENT, USED_MEM_HIGH = 7, 8   # CUmemPool_attribute

    def __init__(self, dev=0):
        self.cu = ctypes.CDLL("libcuda.so.1")
        self.pool = ctypes.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(ctypes.byref(self.pool), ctypes.c_int(dev)) == 0

    def _get(self, attr):
        v = ctypes.c_uint64()
        assert self.cu.cuMemPoolGetAttribute(self.pool, ctypes.c_int(attr), ctypes.byref(v)) == 0
        return v.value

    def reset(self):
        zero = ctypes.c_uint64(0)   # resets the high-water mark to the current use
        assert self.cu.cuMemPoolSetAttribute(self.pool, ctypes.c_int(self.USED_MEM_HIGH), ctypes.byref(zero)) == 0
        return self._get(self.USED_MEM_CURRENT)

    def high(self):
        return self._get(self.USED_MEM_HIGH)


def call_noalloc(builder, plan, x, y, out=None):
    if builder._swap_operands:
        x, y = y, x
    if out is None:
        out = torch.empty(builder.recipe["out_shape"], dtype=torch.float32, device="cuda")
    rc = lib().pe_contract_noalloc(ctypes.byref(plan), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                   ctypes.c_void_p(out.data_ptr()),
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, out


# scratch users: split-K partials (long K, few tiles), the thin kernel's chunk
# partials (matrix-vector product, 64 chunks per output), gathered operands
CASES = [("ts, sp -> tp", (512, 8192), (8192, 128), torch.float32),
         ("ij, j -> i", (64, 1 << 16), (1 << 16,), torch.float32),
         ("bhsc, bcht -> bsht", (2, 8, 16, 20), (2, 20, 8, 24), torch.float16),  # 40-byte rows: gathered
         ("bij, bjk -> bik", (2, 128, 8192), (2, 8192, 96), torch.float16),
         ("ij, jk -> ik", (64, 64), (64, 64), torch.float16)]


@pytest.mark.parametrize("eq,s0,s1,dtype", CASES)
def test_noalloc_matches_pe_contract_twice(eq, s0, s1, dtype):
    b = EinsumBuilder(eq, [s0, s1], dtype)
    run = b.build()
    plan = plan_of(b)
    tol_dtype = dtype
    pool = PoolUsage(torch.cuda.current_device())
    for k in range(2):  # two calls in a row: the shared array is reused
        x, y = seeded(s0, dtype, 70 + k, "randn").cuda(), seeded(s1, dtype, 80 + k, "randn").cuda()
        ref = run(x, y)
        out = torch.empty(b.recipe["out_shape"], dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        used = pool.reset()
        rc, out = call_noalloc(b, plan, x, y, out)
        assert rc == 0, _core.error_string(rc)
        torch.cuda.synchronize()
        assert pool.high() == used, "pe_contract_noalloc allocated from the stream-ordered pool"
        check_close(out, ref.cpu().numpy(), tol_dtype)
        check_close(out, oracle.einsum_cpu(eq, x.cpu(), y.cpu()), tol_dtype)
    assert _core.device_error(torch.cuda.current_stream().cuda_stream) == 0
    b.cleanup()


def test_noalloc_rejects_oversized_scratch():
    # fp16 rows of 20 elements (40 bytes) cannot be read by a tensor map, so the
    # operand is gathered: 1M x 24 x 2 bytes = 48 MB > the 32 MiB array.
    eq, s0, s1 = "ij, jk -> ik", (1 << 20, 20), (20, 64)
    b = EinsumBuilder(eq, [s0, s1], torch.float16)
    b.build()
    assert lib().pe_noalloc_scratch_bytes() == 32 << 20
    x = torch.zeros(s0, dtype=torch.float16, device="cuda")
    y = torch.zeros(s1, dtype=torch.float16, device="cuda")
    rc, _ = call_noalloc(b, plan_of(b), x, y)
    assert rc == 5  # PE_ERR_WORKSPACE
    b.cleanup()
