"""Every BASELINE config at its full size on one GPU against the CPU oracle.

The corpus tests pin each kernel variant on small shapes; these pin the
configurations themselves (index widths, tile-count edges, the fused bsht
store at scale, config 3u's ragged tiles), through the public EinsumBuilder
path, in the comparison structure of the reference's tests/test_einsum.py:131-154.
Contractions are compared on slices covering every tile class of the launch
(relative Frobenius <= 1e-5 fp32, <= 2e-3 fp16 in / fp32 out); the streaming
multiplies must match the whole output bit for bit.
"""
import os

import pytest
import torch

import fullsize
from pto_einsum import EinsumBuilder, _core

pytestmark = pytest.mark.gpu

NAMES = [n for n in fullsize.CFG]
THREADS = min(os.cpu_count() or 1, 32)


@pytest.mark.parametrize("name", NAMES)
def test_config_full_size_matches_oracle(name):
    eq, s0, s1, dt = fullsize.CFG[name]
    a, b = fullsize.make_inputs(name)
    dev = torch.device("cuda", 0)
    bld = EinsumBuilder(eq, [s0, s1], getattr(torch, dt), device=dev)
    run = bld.build()
    out = run(a.to(dev), b.to(dev))
    again = run(a.to(dev), b.to(dev))
    assert _core.device_error(torch.cuda.current_stream(dev).cuda_stream) == 0
    assert torch.equal(out, again), "two calls on the same inputs differ"
    res = fullsize.check(name, a, b, out.cpu(), threads=THREADS)
    if name in fullsize.EXACT:
        assert res["bit_exact"], res
    else:
        assert res["rel_frobenius"] <= fullsize.TOL[dt], res
    bld.cleanup()
