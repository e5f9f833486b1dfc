"""Generate the golden fixtures from the reference implementation itself.

Run where the reference checkout is present (its path in PTO_EINSUM_REFERENCE,
or the default below):

    python tests/golden/make_golden.py

It imports the reference's own planner (src/pto_einsum/builder.py, with an
empty stand-in for the Ascend-only ``torch_npu`` module that builder.py:10
imports but the planner never uses) and its CPU path (device="cpu": the
reference's templates + include/cpu_einsum.h compiled by its own g++ command,
builder.py:685-736), and writes:

  recipes.json     reference recipes for every corpus case and BASELINE
                   config: device="npu" semantics (the accelerator planner
                   this project mirrors) and device="cpu" semantics, the
                   operand-swap decision, tile_k / split-K gates, and the
                   error text when the planner rejects a case.
  cpu_outputs.npz  for every small corpus case: the seed of its fp32 inputs
                   (numpy default_rng(seed).random, float32) and the output of
                   the reference CPU path, stored whole when small and as
                   checksums (float64 sum, sum of squares, 512 sampled
                   elements) otherwise.

Nothing at test time reads the reference checkout: tests use these files.
"""
import json
import os
import sys
import tempfile
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from corpus import ALL_SMALL, BATCHED_PARTIAL, CONFIGS, case_id  # noqa: E402

REF = os.environ.get("PTO_EINSUM_REFERENCE")  # the reference checkout (required)
FULL_LIMIT = 8192        # outputs up to this many elements are stored whole
N_SAMPLES = 512


def load_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "src")):
        raise SystemExit("set PTO_EINSUM_REFERENCE to the reference checkout (the directory holding src/)")
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    sys.path.insert(0, os.path.join(REF, "src"))
    from pto_einsum import builder as ref_builder  # noqa: E402
    return ref_builder


def jsonable(x):
    if isinstance(x, dict):
        return {k: jsonable(v) for k, v in x.items()}
    if isinstance(x, (tuple, list)):
        return [jsonable(v) for v in x]
    if isinstance(x, (np.integer,)):
        return int(x)
    if isinstance(x, (np.bool_,)):
        return bool(x)
    return x


def recipe_record(ref, eq, s0, s1, device, dtype):
    import torch
    b = ref.EinsumBuilder(eq, [s0, s1], dtype, device=device)
    rec = {}
    try:
        b.parse_equation()
        rec["recipe"] = jsonable(dict(b.recipe))
        rec["swap"] = bool(b._swap_operands)
        if not b.recipe["elementwise"] and not b.recipe["broadcast"]:
            tile = int(os.getenv("EINSUM_TILE_SIZE", "128"))
            r = b.recipe
            rec["tile_k"] = int(b._tile_k(tile, r["L0"], r["L1"], r["C"]))
            rec["splitk"] = bool(b._splitk_eligible())
    except (ValueError, TypeError) as e:
        rec["error"] = f"{type(e).__name__}: {e}"
        try:
            rec["recipe_unguarded"] = jsonable(dict(b.parse_recipe(eq, s0, s1)))
        except (ValueError, TypeError) as e2:
            rec["recipe_unguarded_error"] = f"{type(e2).__name__}: {e2}"
    del torch
    return rec


def run_reference_cpu(ref, eq, a, b, build_dir):
    """The reference CPU path; the batched partial-tile guard is bypassed the
    same way its CPU kernel would run (cpu_einsum.h has no tile restriction)."""
    import ctypes
    import torch
    os.environ["EINSUM_BUILD_DIR"] = build_dir
    ta, tb = torch.from_numpy(a), torch.from_numpy(b)
    bld = ref.EinsumBuilder(eq, [ta.shape, tb.shape], torch.float32, device="cpu")
    try:
        run = bld.build()
        return run(ta, tb).numpy()
    except ValueError as e:
        if "Partial tiles" not in str(e):
            raise
    bld.recipe = bld.parse_recipe(eq, tuple(ta.shape), tuple(tb.shape))
    bld._exec_shapes = (tuple(ta.shape), tuple(tb.shape))
    bld.generate_code()
    bld.compile()
    bld.load_library()
    out = torch.zeros(bld.recipe["out_shape"], dtype=torch.float32)
    P = ctypes.POINTER
    bld.lib.run_einsum(ctypes.cast(ta.data_ptr(), P(ctypes.c_float)), ctypes.cast(tb.data_ptr(), P(ctypes.c_float)),
                       ctypes.cast(out.data_ptr(), P(ctypes.c_float)), None)
    return out.numpy()


def inputs_for(seed, s0, s1):
    rng = np.random.default_rng(seed)
    a = rng.random(s0, dtype=np.float32)
    b = rng.random(s1, dtype=np.float32)
    return a, b


def sample_index(n, k=N_SAMPLES):
    return np.unique(np.linspace(0, n - 1, num=min(k, n)).astype(np.int64))


def main():
    import torch
    ref = load_reference()
    recipes = {}
    cases = [(eq, s0, s1, "float32") for eq, s0, s1 in ALL_SMALL] + \
            [(eq, s0, s1, dt) for _, eq, s0, s1, dt in CONFIGS]
    for eq, s0, s1, dt in cases:
        key = case_id(eq, s0, s1)
        dtype = getattr(torch, dt)
        recipes[key] = {
            "equation": eq, "shape0": list(s0), "shape1": list(s1), "dtype": dt,
            "npu": recipe_record(ref, eq, tuple(s0), tuple(s1), "npu", dtype),
            "cpu": recipe_record(ref, eq, tuple(s0), tuple(s1), "cpu", torch.float32),
        }
    with open(os.path.join(HERE, "recipes.json"), "w") as f:
        json.dump(recipes, f, indent=1, sort_keys=True)

    arrays = {}
    with tempfile.TemporaryDirectory() as bd:
        for idx, (eq, s0, s1) in enumerate(ALL_SMALL):
            key = case_id(eq, s0, s1)
            seed = 1000 + idx
            a, b = inputs_for(seed, s0, s1)
            out = run_reference_cpu(ref, eq, a, b, bd)
            flat = out.astype(np.float64).ravel()
            arrays[f"{key}::seed"] = np.array([seed], dtype=np.int64)
            arrays[f"{key}::shape"] = np.array(out.shape, dtype=np.int64)
            arrays[f"{key}::sum"] = np.array([flat.sum(), (flat * flat).sum()], dtype=np.float64)
            if out.size <= FULL_LIMIT:
                arrays[f"{key}::out"] = out.astype(np.float32)
            else:
                idx_s = sample_index(out.size)
                arrays[f"{key}::sidx"] = idx_s
                arrays[f"{key}::sval"] = out.ravel()[idx_s].astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "cpu_outputs.npz"), **arrays)
    print(f"wrote {len(recipes)} recipes, {len(ALL_SMALL)} CPU outputs; partial-guard cases: "
          f"{[case_id(*c) for c in BATCHED_PARTIAL]}")


if __name__ == "__main__":
    main()
