"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

from oracle import oracle

TOL = {torch.float32: 1e-5, torch.float16: 2e-3}   # relative Frobenius vs the CPU oracle


def seeded(shape, dtype, seed, kind="rand"):
    g = torch.Generator().manual_seed(seed)
    if kind == "rand":
        x = torch.rand(shape, generator=g, dtype=torch.float32)
    else:
        x = torch.randn(shape, generator=g, dtype=torch.float32)
    return x.to(dtype)


def check_close(out, ref, dtype, exact=False):
    out = out.detach().float().cpu().numpy() if isinstance(out, torch.Tensor) else out
    assert out.shape == ref.shape, (out.shape, ref.shape)
    if exact:
        np.testing.assert_array_equal(out, ref)
        return 0.0
    assert np.isfinite(out).all()
    err = oracle.rel_frobenius(out, ref)
    assert err <= TOL[dtype], f"relative Frobenius error {err:.3e} > {TOL[dtype]:.0e}"
    return err
