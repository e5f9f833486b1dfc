"""Pin the CPU oracle (oracle/oracle.py + einsum_oracle.c) to the reference.

The golden outputs were produced by the reference's own CPU path
(tests/golden/make_golden.py). The oracle follows the same accumulation order,
so agreement is bit-exact.
"""
import json
import os

import numpy as np
import pytest

from corpus import ALL_SMALL, case_id
from oracle import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
OUT = np.load(os.path.join(GOLD, "cpu_outputs.npz"))
with open(os.path.join(GOLD, "recipes.json")) as f:
    RECIPES = json.load(f)


def golden_inputs(key, s0, s1):
    seed = int(OUT[f"{key}::seed"][0])
    rng = np.random.default_rng(seed)
    return rng.random(s0, dtype=np.float32), rng.random(s1, dtype=np.float32)


def check_against_golden(key, out):
    assert tuple(out.shape) == tuple(OUT[f"{key}::shape"])
    if f"{key}::out" in OUT:
        np.testing.assert_array_equal(out, OUT[f"{key}::out"])
    else:
        idx = OUT[f"{key}::sidx"]
        np.testing.assert_array_equal(out.ravel()[idx], OUT[f"{key}::sval"])
    flat = out.astype(np.float64).ravel()
    s, ss = OUT[f"{key}::sum"]
    assert flat.sum() == pytest.approx(s, rel=1e-12, abs=1e-9)
    assert (flat * flat).sum() == pytest.approx(ss, rel=1e-12, abs=1e-9)


@pytest.mark.parametrize("eq,s0,s1", ALL_SMALL, ids=[case_id(*c) for c in ALL_SMALL])
def test_oracle_matches_reference_cpu(eq, s0, s1):
    key = case_id(eq, s0, s1)
    a, b = golden_inputs(key, s0, s1)
    check_against_golden(key, oracle.einsum_cpu(eq, a, b))


@pytest.mark.parametrize("eq,s0,s1", ALL_SMALL[:20], ids=[case_id(*c) for c in ALL_SMALL[:20]])
def test_oracle_threads_do_not_change_bits(eq, s0, s1):
    key = case_id(eq, s0, s1)
    a, b = golden_inputs(key, s0, s1)
    np.testing.assert_array_equal(oracle.einsum_cpu(eq, a, b, threads=1), oracle.einsum_cpu(eq, a, b, threads=4))


@pytest.mark.parametrize("key", sorted(RECIPES))
def test_oracle_cpu_plan_matches_reference(key):
    case = RECIPES[key]
    rec = case["cpu"]
    r = rec.get("recipe") or rec.get("recipe_unguarded")
    if r is None:
        pytest.skip("rejected by the reference planner")
    plan = oracle.cpu_plan(case["equation"], case["shape0"], case["shape1"])
    if r["elementwise"]:
        assert plan["elementwise"]
        return
    if rec.get("swap"):
        # the reference planned the swapped operand order; the oracle keeps the
        # natural order (products commute, the c order is the same)
        return
    assert list(plan["perm0"]) == r["in_transpose_idxs"][0]
    assert list(plan["perm1"]) == r["in_transpose_idxs"][1]
    assert list(plan["out_perm"]) == r["out_transpose_idxs"]
    assert (plan["I"], plan["L0"], plan["L1"], plan["C"]) == (r["I"], r["L0"], r["L1"], r["C"])


def test_broadcast_definition_matches_matmul_route():
    # device='cpu' routes broadcasts through the matmul path (builder.py:373-376);
    # the broadcast definition used for the CUDA route gives the same bits.
    from pto_einsum import planner
    rng = np.random.default_rng(7)
    for eq, s0, s1 in [("bsd,d->bsd", (2, 8, 64), (64,)), ("bshd,sd->bshd", (2, 8, 4, 16), (8, 16)),
                       ("hqk,h->hqk", (8, 16, 16), (8,)), ("bsd,sd->bsd", (2, 8, 64), (8, 64)),
                       ("h,hqk->hqk", (8,), (8, 16, 16))]:
        a, b = rng.standard_normal(s0).astype(np.float32), rng.standard_normal(s1).astype(np.float32)
        r, _ = planner.choose_operand_order("cuda", eq, s0, s1)
        assert r["broadcast"]
        np.testing.assert_array_equal(oracle.broadcast_cpu(r, a, b), oracle.einsum_cpu(eq, a, b))


def test_reference_library_agrees_with_oracle():
    """oracle/_ref holds the reference's CPU libraries compiled from its own
    sources (oracle/build_ref.py); when present they must match bit for bit."""
    from oracle import ref_cpu
    if not ref_cpu.available():
        pytest.skip("oracle/_ref not built")
    for name in ref_cpu.names():
        spec = ref_cpu.spec(name)
        a, b = ref_cpu.sample_inputs(name, seed=3)
        np.testing.assert_array_equal(ref_cpu.run(name, a, b), oracle.einsum_cpu(spec["equation"], a, b))
