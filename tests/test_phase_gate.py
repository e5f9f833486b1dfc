"""EINSUM_PHASE_STOP on the GPU: the reference's phase-profiling gate
(include/pto_einsum.h:18-30) as built here. A library generated with
EINSUM_EXTRA_DEFINES="-DEINSUM_PHASE_STOP=N" still launches the fused kernel
(the launch and pipeline-barrier skeleton is kept), but below 3 it writes no
output; at 3 it is the ordinary contraction. Each level is timed too, and the
times must not shrink as phases are added back (within noise)."""

import pytest
import torch

from gpu_util import check_close, seeded
from oracle import oracle
from pto_einsum import EinsumBuilder, _core

pytestmark = pytest.mark.gpu

CASES = [
    ("bij, bjk -> bik", (4, 512, 1024), (4, 1024, 512), torch.float16),     # CTA pairs
    ("bshd, bthd -> bsht", (2, 256, 4, 80), (2, 200, 4, 80), torch.float16),  # fused permuted store
    ("tn, sn -> ts", (1024, 128), (1024, 128), torch.float32),               # 3xTF32, pre-pass
    ("ts, sp -> tp", (512, 8192), (8192, 128), torch.float32),               # split-K / stream-K
    ("bhsc, bcht -> bsht", (2, 8, 16, 20), (2, 20, 8, 24), torch.float16),   # gathered operand
]


def _build(eq, s0, s1, dt, stop, monkeypatch):
    monkeypatch.setenv("EINSUM_EXTRA_DEFINES", f"-DEINSUM_PHASE_STOP={stop}")
    b = EinsumBuilder(eq, [s0, s1], dt)
    run = b.build()
    return b, run


@pytest.mark.parametrize("eq,s0,s1,dt", CASES)
def test_phase_levels(eq, s0, s1, dt, monkeypatch):
    x, y = seeded(s0, dt, 5, "randn").cuda(), seeded(s1, dt, 6, "randn").cuda()
    stream = torch.cuda.current_stream().cuda_stream
    times = []
    for stop in (0, 1, 2, 3):
        b, run = _build(eq, s0, s1, dt, stop, monkeypatch)
        out = torch.full(b.recipe["out_shape"], float("nan"), device="cuda")
        ws = b.workspace(torch.device("cuda", torch.cuda.current_device()), stream)
        p0, p1 = (y, x) if b._swap_operands else (x, y)
        n0 = _core.launch_count()
        b.lib.run_einsum_exec(p0.data_ptr(), p1.data_ptr(), out.data_ptr(), ws, stream)
        assert b.lib.run_einsum_last_error() == 0
        torch.cuda.synchronize()
        assert _core.launch_count() > n0, "the fused kernel must still launch"
        assert _core.device_error(stream) == 0
        if stop < 3:
            assert torch.isnan(out).all(), f"stop={stop} wrote output"
        else:
            check_close(out, oracle.einsum_cpu(eq, x.cpu(), y.cpu()), dt)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for _ in range(3):
            b.lib.run_einsum_exec(p0.data_ptr(), p1.data_ptr(), out.data_ptr(), ws, stream)
        ev[0].record()
        for _ in range(20):
            b.lib.run_einsum_exec(p0.data_ptr(), p1.data_ptr(), out.data_ptr(), ws, stream)
        ev[1].record()
        torch.cuda.synchronize()
        times.append(ev[0].elapsed_time(ev[1]) / 20)
        b.cleanup()
    monkeypatch.delenv("EINSUM_EXTRA_DEFINES")
    # adding phases back never makes the kernel much faster (2 us or 25% slack)
    for lo, hi in zip(times, times[1:]):
        assert hi >= min(lo * 0.75, lo - 0.002), times
