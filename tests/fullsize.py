"""BASELINE configs at their full sizes: seeded inputs and sampled parity.

Shared by the full-size GPU parity tests and bench.py's `parity` fields.

Inputs follow the distributions the configs name: U[0,1) for config 2,
N(0,1) for configs 3 and 4, the lower-triangular decay mask
D[t,s] = 0.99^(t-s) (s <= t, else 0) for 4b, and the rms weight, RoPE
cos/sin table and ALiBi slopes for config 5. Every tensor is generated on the
CPU from a seeded generator, so a sharded run's shards concatenate to the
single-device tensors.

Parity at full size compares the CUDA result with the CPU oracle (a
restatement of the reference's include/cpu_einsum.h:53-92) on slices that
cover every tile class of the full launch: first and last batch (config 2),
first and last (b, h) pair with config 3u's ragged last row and column tiles
inside them (configs 3 / 3u), first and last 512-row slab (4a, 4c), and the
whole output bit for bit for the streaming multiplies (4b, 5). A slice of a
label narrows that axis in every operand that carries it and in the output,
so the sliced equation is the same equation on smaller operands.
"""
from __future__ import annotations

import numpy as np
import torch

from corpus import CONFIGS

CFG = {name: (eq, s0, s1, dt) for name, eq, s0, s1, dt in CONFIGS}
TOL = {"float32": 1e-5, "float16": 2e-3}   # relative Frobenius vs the CPU oracle
EXACT = {"cfg4b", "cfg5_rms", "cfg5_rope", "cfg5_alibi"}


def labels(eq):
    lhs, out = eq.replace(" ", "").split("->")
    a, b = lhs.split(",")
    return a, b, out


def make_inputs(name, seed=1000, device="cpu"):
    """Seeded inputs of config `name` (fp16 or fp32 as the config says),
    generated on `device` from a generator of that device."""
    eq, s0, s1, dt = CFG[name]
    dtype = getattr(torch, dt)
    g = torch.Generator(device=device).manual_seed(seed)
    kw = dict(device=device)
    if name in ("cfg1", "cfg2"):
        a = torch.rand(s0, generator=g, dtype=torch.float32, **kw)
        b = torch.rand(s1, generator=g, dtype=torch.float32, **kw)
    elif name == "cfg4b":
        a = torch.randn(s0, generator=g, dtype=torch.float32, **kw)
        t = torch.arange(s0[0], dtype=torch.float32, **kw)
        sv = torch.arange(s0[1], dtype=torch.float32, **kw)
        diff = t[:, None] - sv[None, :]
        b = torch.where(diff >= 0, torch.pow(torch.tensor(0.99, **kw), diff.clamp(min=0)),
                        torch.zeros((), **kw))
    elif name == "cfg5_rms":
        a = torch.randn(s0, generator=g, **kw)
        b = torch.rand(s1, generator=g, **kw) + 0.5
    elif name == "cfg5_rope":
        a = torch.randn(s0, generator=g, **kw)
        S, D = s1
        pos = torch.arange(S, dtype=torch.float64)[:, None]
        j = torch.arange(D // 2, dtype=torch.float64)[None, :]
        ang = pos * torch.pow(10000.0, -2.0 * j / D)
        b = torch.cat([torch.cos(ang), torch.sin(ang)], dim=1).float().to(device)
    elif name == "cfg5_alibi":
        a = torch.randn(s0, generator=g, **kw)
        H = s1[0]
        b = torch.pow(2.0, -8.0 * (torch.arange(H, dtype=torch.float64) + 1) / H).float().to(device)
    else:
        a = torch.randn(s0, generator=g, **kw)
        b = torch.randn(s1, generator=g, **kw)
    return a.to(dtype).contiguous(), b.to(dtype).contiguous()


def slices(name, out_shape, whole_exact=True):
    """Selections {label: (lo, hi)} whose union covers every tile class of the
    full-size launch; None = the whole output. With whole_exact=False the
    streaming multiplies are checked on their first and last leading index
    only (the bench's quicker sample; the tests check the whole output)."""
    eq = CFG[name][0]
    _, _, o = labels(eq)
    size = dict(zip(o, out_shape))
    if name == "cfg1" or (name in EXACT and whole_exact):
        return [None]
    if name in EXACT:
        lead = o[0]
        return [{lead: (0, 1)}, {lead: (size[lead] - 1, size[lead])}]
    if name == "cfg2":
        return [{"b": (0, 1)}, {"b": (size["b"] - 1, size["b"])}]
    if name in ("cfg3", "cfg3u"):
        return [{"b": (0, 1), "h": (0, 1)},
                {"b": (size["b"] - 1, size["b"]), "h": (size["h"] - 1, size["h"])}]
    if name in ("cfg4a", "cfg4c"):
        t = size["t"]
        w = min(512, t)
        return [{"t": (0, w)}, {"t": (t - w, t)}]
    raise KeyError(name)


def _narrow(x, lab, sel):
    for ch, (lo, hi) in sel.items():
        if ch in lab:
            x = x.narrow(lab.index(ch), lo, hi - lo)
    return x


def check(name, a, b, out, threads=8, whole_exact=True):
    """Compare `out` (CUDA result of config `name` on CPU inputs a, b) with the
    oracle on the config's covering slices. Returns dict(rel_frobenius=max over
    slices, bit_exact=all slices identical, slices=[...])."""
    from oracle import oracle
    eq = CFG[name][0]
    la, lb, lo = labels(eq)
    out = out.detach()
    worst, exact, desc = 0.0, True, []
    for sel in slices(name, tuple(out.shape), whole_exact):
        if sel is None:
            x, y, got = a, b, out
            desc.append("whole output")
        else:
            x, y, got = _narrow(a, la, sel), _narrow(b, lb, sel), _narrow(out, lo, sel)
            desc.append(",".join(f"{k}[{v0}:{v1}]" for k, (v0, v1) in sel.items()))
        ref = oracle.einsum_cpu(eq, x.contiguous(), y.contiguous(), threads=threads)
        g = got.float().cpu().contiguous().numpy()
        assert g.shape == ref.shape, (g.shape, ref.shape)
        exact = exact and bool(np.array_equal(g, ref))
        worst = max(worst, oracle.rel_frobenius(g, ref) if np.isfinite(g).all() else float("inf"))
    return {"rel_frobenius": worst, "bit_exact": exact, "slices": desc}
