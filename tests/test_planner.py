"""Plan identity: pto_einsum.planner must reproduce the reference recipe for
every corpus case and BASELINE config (recipes.json was written by the
reference planner itself, tests/golden/make_golden.py)."""
import json
import os

import pytest
import torch

from pto_einsum import EinsumBuilder, planner

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "recipes.json")
with open(GOLDEN) as f:
    RECIPES = json.load(f)


def norm(r):
    return json.loads(json.dumps(r))  # tuples -> lists, same as the fixture


@pytest.mark.parametrize("key", sorted(RECIPES))
@pytest.mark.parametrize("sem", ["npu", "cpu"])
def test_recipe_identity(key, sem):
    case = RECIPES[key]
    rec = case[sem]
    eq, s0, s1 = case["equation"], tuple(case["shape0"]), tuple(case["shape1"])
    device = "cpu" if sem == "cpu" else "cuda"
    recipe, swapped = planner.choose_operand_order(device, eq, s0, s1)
    guard = planner.partial_tile_message(recipe)
    if "error" in rec:
        # the reference rejected it: either the partial-tile guard (lifted on CUDA,
        # reproduced by partial_tile_message) or a planner error
        if "Partial tiles" in rec["error"]:
            assert guard is not None and guard in rec["error"]
            assert norm(planner.parse_recipe(device, eq, s0, s1)) == rec["recipe_unguarded"]
        else:
            pytest.fail(f"reference raised {rec['error']} but planner accepted")
        return
    assert guard is None
    assert swapped == rec["swap"]
    assert norm(recipe) == rec["recipe"]
    if "tile_k" in rec:
        es = 2 if case["dtype"] == "float16" and sem == "npu" else 4
        t = planner.tile_size()
        assert planner.tile_k(es, t, recipe["L0"], recipe["L1"], recipe["C"]) == rec["tile_k"]
        assert planner.splitk_eligible(recipe, es) == rec["splitk"]


def test_direct_read_gates():
    # the reference's proven-teeth gates (tests/test_einsum.py:291,321,351,388)
    cases = [("bihd, bjhd -> bihj", (2, 128, 16, 128), "in_nt", 1),
             ("bihj, bjhd -> bihd", (2, 128, 16, 128), "in_nt", 2),
             ("bvhd, bvhe -> bhde", (2, 128, 16, 128), "in_nt", 3),
             ("bshd, bthd -> bsht", (2, 128, 4, 64), "out_fusible", 1),
             ("ij, jk -> ik", None, "out_fusible", 0)]
    for eq, s, field, val in cases:
        shapes = [(32, 64), (64, 128)] if s is None else [s, s]
        b = EinsumBuilder(eq, shapes, torch.float32)
        b.parse_equation()
        assert b.recipe[field] == val


def test_env_knobs(monkeypatch):
    monkeypatch.setenv("EINSUM_DISABLE_NT", "1")
    r = planner.parse_recipe("cuda", "bihd,bjhd->bihj", (2, 128, 16, 128), (2, 128, 16, 128))
    assert r["in_nt"] == 0
    monkeypatch.delenv("EINSUM_DISABLE_NT")
    monkeypatch.setenv("EINSUM_DISABLE_OPERAND_SWAP", "1")
    _, sw = planner.choose_operand_order("cuda", "ij,jk->ki", (32, 64), (64, 48))
    assert not sw
    monkeypatch.delenv("EINSUM_DISABLE_OPERAND_SWAP")
    _, sw = planner.choose_operand_order("cuda", "ij,jk->ki", (32, 64), (64, 48))
    assert sw
    monkeypatch.setenv("EINSUM_TILE_SIZE", "64")
    r = planner.parse_recipe("cuda", "bihd,bjhd->bihj", (2, 96, 4, 32), (2, 96, 4, 32))
    assert r["in_nt"] == 0  # 96 is a whole tile at 128 but not a multiple of 64
    monkeypatch.delenv("EINSUM_TILE_SIZE")
    r = planner.parse_recipe("cuda", "bihd,bjhd->bihj", (2, 96, 4, 32), (2, 96, 4, 32))
    assert r["in_nt"] == 1


def test_validation_messages():
    with pytest.raises(ValueError, match="subscripts should be in"):
        planner.validate_expr("i1,jk->ik", (2, 2), (2, 2))
    with pytest.raises(ValueError, match="multiple times"):
        planner.validate_expr("ii,jk->ik", (2, 2), (2, 2))
    with pytest.raises(ValueError, match="not found in inputs"):
        planner.validate_expr("ij,jk->iz", (2, 2), (2, 2))
    with pytest.raises(ValueError, match="Input0 requires 2 dimensions"):
        planner.validate_expr("ij,jk->ik", (2,), (2, 2))
    with pytest.raises(ValueError, match="size mismatches"):
        planner.validate_expr("ij,jk->ik", (2, 3), (4, 2))
    with pytest.raises(ValueError, match="single-operand reduction is not supported"):
        planner.parse_recipe("cuda", "ij,jk->k", (32, 64), (64, 128))


def test_unsupported_dtype_and_cpu_float16():
    b = EinsumBuilder("ij,jk->ik", [(32, 64), (64, 32)], torch.bfloat16)
    b.parse_equation()
    with pytest.raises(TypeError, match="Unsupported torch dtype"):
        b.generate_code()
    c = EinsumBuilder("ij,jk->ik", [(32, 64), (64, 32)], torch.float16, device="cpu")
    c.parse_equation()  # planning works for every device
    with pytest.raises(TypeError, match="float16 is not supported on CPU"):
        c.generate_code()
