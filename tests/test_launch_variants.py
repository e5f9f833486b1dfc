"""Kernel variants selected by environment switches, and dependent back-to-back calls.

The contraction kernel has three switches that a caller can flip and that the
default parity suites do not reach:
  PE_GEMM_KB   1 or 2 contraction rows (128 bytes each) per pipeline stage
  PE_EPI_V8    full-line (32-byte) epilogue stores on / off
  PE_GEMM_PDL  programmatic dependent launch on / off
  PE_EPI_WARPS_PAIR  4 or 8 epilogue warps on fp16 CTA pairs
  PE_GEMM_FUSEB  fp32 fused-B MMAs on / off (changes the accumulation split:
                 compared with the oracle tolerance, not bit for bit)
The first four do not change the order of the tensor-core accumulation, so
those variants must reproduce the default result bit for bit. Each variant runs in a
child process (the switches are read once per process) on the same seeded
inputs; the default run is also checked against a float64 torch.einsum on
the GPU (the CPU-oracle parity of these paths is covered by the parity suites).

Programmatic dependent launch lets a contraction's prologue overlap the
previous kernel. A chained caller whose next contraction reads the previous
output must still see it complete: the chain test issues dependent calls back
to back with no synchronisation and compares with the same chain run one call
at a time.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)

CHILD = r"""
import sys, numpy as np, torch
sys.path[:0] = [{pkg!r}, {repo!r}, {tests!r}]
from pto_einsum import EinsumBuilder
from gpu_util import seeded
cases = [
    ("bij,bjk->bik", (8, 1024, 1024), (8, 1024, 1024), torch.float16),  # CTA pairs, MN-major B
    ("bij,bkj->bik", (8, 1024, 512), (8, 1024, 512), torch.float16),    # CTA pairs, K-major B
    ("bshd,bthd->bsht", (2, 256, 8, 64), (2, 320, 8, 64), torch.float16),  # single CTAs, permuted store
    ("tn,sn->ts", (1024, 128), (1024, 128), torch.float32),            # 3xTF32
    ("ts,sp->tp", (512, 4096), (4096, 128), torch.float32),            # 3xTF32 fused B, stream-K
    ("ij,jk->ik", (300, 200), (200, 520), torch.float16),              # ragged tiles
]
out = {{}}
for k, (eq, s0, s1, dt) in enumerate(cases):
    a = seeded(s0, dt, 500 + k, "randn").cuda()
    b = seeded(s1, dt, 600 + k, "randn").cuda()
    run = EinsumBuilder(eq, [list(s0), list(s1)], dt).build()
    out[str(k)] = run(a, b).cpu().numpy()
torch.cuda.synchronize()
np.savez({path!r}, **out)
"""

VARIANTS = [
    {},
    {"PE_GEMM_KB": "1"},
    {"PE_GEMM_KB": "2"},
    {"PE_EPI_V8": "0"},
    {"PE_EPI_V8": "1"},
    {"PE_GEMM_PDL": "0"},
    {"PE_EPI_WARPS_PAIR": "4"},
    {"PE_EPI_WARPS_PAIR": "8"},
]


def _run_child(env_extra, path):
    code = CHILD.format(pkg=os.path.join(REPO, "pto-einsum_b200"), repo=REPO, tests=HERE, path=path)
    env = dict(os.environ)
    for k in ("PE_GEMM_KB", "PE_EPI_V8", "PE_GEMM_PDL", "PE_GEMM_FUSEB", "PE_EPI_WARPS_PAIR"):
        env.pop(k, None)
    env.update(env_extra)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return dict(np.load(path))


@pytest.mark.gpu
def test_switch_variants_bit_identical(tmp_path):
    from gpu_util import seeded, TOL
    import re
    base = _run_child({}, str(tmp_path / "default.npz"))
    # the default run against float64 on the GPU
    cases = re.findall(r'\("([^"]+)", (\([^)]*\)), (\([^)]*\)), torch\.(float\d+)\)', CHILD)
    assert len(cases) == len(base)
    for k, (eq, s0, s1, dt) in enumerate(cases):
        dt = getattr(torch, dt)
        a = seeded(eval(s0), dt, 500 + k, "randn").cuda().double()
        b = seeded(eval(s1), dt, 600 + k, "randn").cuda().double()
        ref = torch.einsum(eq, a, b)
        got = torch.from_numpy(base[str(k)]).cuda().double()
        err = ((got - ref).norm() / ref.norm()).item()
        assert err <= TOL[dt], (eq, err)
    for j, v in enumerate(VARIANTS[1:]):
        got = _run_child(v, str(tmp_path / f"v{j}.npz"))
        for key in base:
            np.testing.assert_array_equal(got[key], base[key], err_msg=f"variant {v}, case {key}")
    # three separate MMAs instead of the fused-B pair: same tolerance as the default
    got = _run_child({"PE_GEMM_FUSEB": "0"}, str(tmp_path / "nofuse.npz"))
    for k, (eq, s0, s1, dt) in enumerate(cases):
        dt = getattr(torch, dt)
        a = seeded(eval(s0), dt, 500 + k, "randn").cuda().double()
        b = seeded(eval(s1), dt, 600 + k, "randn").cuda().double()
        ref = torch.einsum(eq, a, b)
        g = torch.from_numpy(got[str(k)]).cuda().double()
        assert ((g - ref).norm() / ref.norm()).item() <= TOL[dt], eq


@pytest.mark.gpu
def test_dependent_calls_back_to_back():
    from pto_einsum import EinsumBuilder
    from gpu_util import seeded
    n = 512
    first = EinsumBuilder("ij,jk->ik", [[n, n], [n, n]], torch.float32).build()
    second = EinsumBuilder("ik,kl->il", [[n, n], [n, n]], torch.float32).build()
    a = seeded((n, n), torch.float32, 11, "randn").cuda()
    bs = [seeded((n, n), torch.float32, 20 + k, "randn").cuda() / 16 for k in range(6)]

    def chain(sync):
        x = a
        for k, b in enumerate(bs):
            x = (first if k % 2 == 0 else second)(x, b)
            if sync:
                torch.cuda.synchronize()
        return x

    ref = chain(True).cpu()
    for _ in range(5):
        got = chain(False)
        torch.cuda.synchronize()
        assert torch.equal(got.cpu(), ref)
