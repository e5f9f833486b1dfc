"""Device-side failure handling without a GPU fault: a pipeline wait that nothing
completes gives up after its limit, records PE_ERR_TIMEOUT in the device error word,
and the kernel returns; the host reads the status and the context stays usable."""
import time

import pytest
import torch

from pto_einsum import _core, einsum

PE_ERR_INVALID, PE_ERR_TIMEOUT = 1, 6


@pytest.mark.gpu
def test_bounded_wait_times_out_and_context_survives():
    lib = _core.core_lib()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.pe_device_error(st) == 0
    t0 = time.perf_counter()
    code = lib.pe_selftest_wait_timeout(2_000_000, st)          # 2 ms limit
    elapsed = time.perf_counter() - t0
    assert code == PE_ERR_TIMEOUT | (15 << 8), code
    assert elapsed < 5.0
    assert lib.pe_device_error(st) == 0                         # read and cleared
    # the context still runs contractions correctly
    g = torch.Generator().manual_seed(3)
    a = torch.rand(256, 384, generator=g).cuda()
    b = torch.rand(384, 128, generator=g).cuda()
    out = einsum("ij,jk->ik", a, b)
    ref = a.double() @ b.double()
    assert ((out.double() - ref).norm() / ref.norm()).item() < 1e-5
    assert lib.pe_device_error(st) == 0


@pytest.mark.gpu
def test_selftest_rejects_long_limits():
    lib = _core.core_lib()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.pe_selftest_wait_timeout(10 ** 9, st) == PE_ERR_INVALID
