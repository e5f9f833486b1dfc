"""Compile the reference's own CPU libraries into oracle/_ref/ (TEST
INFRASTRUCTURE ONLY; run in a container where the reference checkout exists).

    python oracle/build_ref.py [--reference <reference checkout>]

For every spec in ref_specs.SPECS this runs the reference planner and code
generator (src/pto_einsum/builder.py:555-683, device="cpu") and its compile
step (builder.py:685-736: g++ -O3 -shared -fPIC -std=c++17 -I include/, i.e.
the reference's templates.py CPU template + include/cpu_einsum.h), with the
build directory pointed at oracle/_ref/build, then copies each library to
oracle/_ref/<name>.so and writes oracle/_ref/manifest.json. The reference's
Ascend-only ``torch_npu`` import (builder.py:10) gets an empty stand-in; the
CPU path never touches it. Nothing is copied from the reference sources into
this repository: the outputs are build products under the git-ignored _ref/.
"""
import argparse
import json
import os
import shutil
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
sys.path.insert(0, HERE)
from ref_specs import SPECS  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PTO_EINSUM_REFERENCE"),
                    help="reference checkout (default: $PTO_EINSUM_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        print("no reference checkout given (--reference or PTO_EINSUM_REFERENCE); oracle/_ref not built")
        return 0
    src = os.path.join(args.reference, "src")
    if not os.path.isdir(src):
        print(f"reference sources not found at {src}; oracle/_ref not built")
        return 1
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    sys.path.insert(0, src)
    import torch
    from pto_einsum import builder as ref  # the reference package
    os.makedirs(OUT, exist_ok=True)
    os.environ["EINSUM_BUILD_DIR"] = os.path.join(OUT, "build")
    manifest = {}
    for name, (eq, s0, s1, units, cfg) in SPECS.items():
        b = ref.EinsumBuilder(eq, [s0, s1], torch.float32, device="cpu")
        b.parse_equation()
        b.generate_code()
        b.compile()
        dst = os.path.join(OUT, f"{name}.so")
        shutil.copyfile(b.so_filename, dst)
        manifest[name] = dict(equation=eq, shape0=list(s0), shape1=list(s1), units=units, config=cfg,
                              out_shape=list(b.recipe["out_shape"]), swap=bool(b._swap_operands))
        print(f"{name}: {dst}")
    shutil.rmtree(os.path.join(OUT, "build"), ignore_errors=True)
    with open(os.path.join(OUT, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
