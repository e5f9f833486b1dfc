"""device="cpu" through the public API (product host path, no GPU).

The reference runs device="cpu" builds on its g++-compiled CPU library
(src/pto_einsum/builder.py:606-626, :704-709, :856-875). This package generates
its own host library from include/pto_einsum_cpu.h; it must reproduce the
reference CPU outputs bit for bit: against the golden outputs written by the
reference itself (tests/golden/cpu_outputs.npz) and against the oracle.
"""
import numpy as np
import pytest
import torch

from corpus import ALL_SMALL, case_id
from oracle import oracle
from pto_einsum import EinsumBuilder, einsum
from test_oracle import check_against_golden, golden_inputs


def test_cpu_backend_whole_corpus_matches_reference_golden():
    """All 72 corpus cases through einsum(..., device="cpu"), bit for bit against
    the outputs of the reference's own CPU path and against the oracle."""
    bad = []
    for eq, s0, s1 in ALL_SMALL:
        key = case_id(eq, s0, s1)
        a, b = golden_inputs(key, s0, s1)
        out = einsum(eq, torch.from_numpy(a), torch.from_numpy(b), device="cpu")
        assert out.device.type == "cpu" and out.dtype == torch.float32
        try:
            check_against_golden(key, out.numpy())
        except AssertionError:
            bad.append(key)
            continue
        if not np.array_equal(out.numpy(), oracle.einsum_cpu(eq, a, b)):
            bad.append(key + " (oracle)")
    assert not bad, bad


def test_config1_on_cpu_path():
    """'ij,jk->ik' fp32 256x256, torch.rand seeded, device='cpu'."""
    g = torch.Generator().manual_seed(0)
    a = torch.rand((256, 256), generator=g)
    b = torch.rand((256, 256), generator=g)
    bld = EinsumBuilder("ij,jk->ik", [a.shape, b.shape], torch.float32, device="cpu")
    run = bld.build()
    out = run(a, b)
    np.testing.assert_array_equal(out.numpy(), oracle.einsum_cpu("ij,jk->ik", a, b))
    exp = (a.double() @ b.double()).float()
    torch.testing.assert_close(out, exp, rtol=1e-5, atol=1e-5)
    assert "in_nt" in bld.cpp_code and bld.so_filename.endswith(".so")
    bld.cleanup()


def test_cpu_large_rows_threads_bit_identical():
    """Large enough to run on several host threads: rows are split among
    threads, each element computed by one thread in the reference order."""
    g = torch.Generator().manual_seed(3)
    a = torch.randn((4, 384, 512), generator=g)
    b = torch.randn((4, 512, 320), generator=g)
    out = einsum("bij,bjk->bik", a, b, device="cpu")
    np.testing.assert_array_equal(out.numpy(), oracle.einsum_cpu("bij,bjk->bik", a, b))


def test_cpu_rejects_float16_like_reference():
    with pytest.raises(TypeError, match="float16 is not supported on CPU"):
        EinsumBuilder("ij,jk->ik", [(4, 4), (4, 4)], torch.float16, device="cpu").build()


def test_cpu_runner_checks_inputs():
    run = EinsumBuilder("ij,jk->ik", [(8, 4), (4, 8)], torch.float32, device="cpu").build()
    with pytest.raises(ValueError, match="do not match built shapes"):
        run(torch.zeros(4, 8), torch.zeros(4, 8))
    with pytest.raises(TypeError, match="do not match built datatype"):
        run(torch.zeros(8, 4, dtype=torch.float64), torch.zeros(4, 8, dtype=torch.float64))


def test_cpu_broadcast_takes_matmul_route():
    """On CPU the reference skips the broadcast classifier (builder.py:373-376):
    'bsd,d->bsd' plans as a matmul with C = 1 and gives the exact products."""
    bld = EinsumBuilder("bsd,d->bsd", [(2, 8, 16), (16,)], torch.float32, device="cpu")
    run = bld.build()
    assert not bld.recipe["broadcast"] and not bld.recipe["elementwise"]
    g = torch.Generator().manual_seed(5)
    x, w = torch.randn((2, 8, 16), generator=g), torch.randn((16,), generator=g)
    assert torch.equal(run(x, w), x * w)
