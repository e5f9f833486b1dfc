"""The C ABI: libraries load and export every symbol the headers declare;
the generated per-equation libraries keep the reference's entry-point names
and the md5-keyed cache behaves like the reference's (no GPU needed)."""
import os
import re
import subprocess

import pytest
import torch

from pto_einsum import EinsumBuilder, _core

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    text = open(os.path.join(REPO, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b((?:pe|run)_\w+)\s*\(", text))


def exported(so):
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_core_library_exports_header():
    lib = _core.core_lib()
    assert lib is not None
    syms = declared("pto_einsum_b200.h")
    assert len(syms) >= 15
    missing = syms - exported(_core.LIB_PATH)
    assert not missing, missing
    assert _core.core_version().startswith("pto_einsum_b200 sm_100a")


ROUTES = [("ij,jk->ik", [(32, 64), (64, 32)], "matmul"),
          ("ts,ts->ts", [(8, 8), (8, 8)], "elementwise"),
          ("bsd,d->bsd", [(2, 8, 64), (64,)], "broadcast")]


@pytest.mark.parametrize("eq,shapes,route", ROUTES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_generated_library_exports(eq, shapes, route, dtype):
    b = EinsumBuilder(eq, shapes, dtype)
    b.parse_equation()
    b.generate_code()
    b.compile()
    b.load_library()
    syms = exported(b.so_filename)
    abi = declared("pto_einsum_abi.h")
    need = {"run_einsum", "run_einsum_setup", "run_einsum_exec", "run_einsum_exec_rc", "run_einsum_teardown",
            "run_einsum_last_error"}
    if route == "matmul":
        need = abi
    assert need <= abi
    assert not (need - syms), need - syms
    b.cleanup()


def test_cache_and_cleanup():
    b = EinsumBuilder("ij, jk -> ik", [(16, 32), (32, 16)], torch.float32)
    b.parse_equation()
    b.generate_code()
    b.compile()
    assert os.path.exists(b.target_dir) and os.path.exists(b.cpp_filename) and os.path.exists(b.so_filename)
    assert os.path.basename(b.target_dir) == b.code_hash
    t = os.path.getmtime(b.so_filename)
    c = EinsumBuilder("ij, jk -> ik", [(16, 32), (32, 16)], torch.float32)
    c.parse_equation()
    c.generate_code()
    c.compile()  # cache hit: same md5, no rebuild
    assert c.so_filename == b.so_filename and os.path.getmtime(c.so_filename) == t
    b.load_library()
    b.cleanup()
    assert not os.path.exists(b.target_dir)


def _undefined_symbols(so):
    out = subprocess.run(["nm", "-D", "--undefined-only", so], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


@pytest.mark.parametrize("stop", [None, 0, 1, 2, 3])
def test_extra_defines_phase_stop_reaches_the_core(monkeypatch, stop):
    """EINSUM_EXTRA_DEFINES carries -DEINSUM_PHASE_STOP=N into the generated
    library (reference builder.py:691-700, profile_phase_overlap.py:72-93): the
    cached file name gets a define tag and, below 3, run_einsum_exec calls the
    phase-gated core entry point instead of the ordinary one."""
    if stop is not None:
        monkeypatch.setenv("EINSUM_EXTRA_DEFINES", f"-DEINSUM_PHASE_STOP={stop}")
    else:
        monkeypatch.delenv("EINSUM_EXTRA_DEFINES", raising=False)
    b = EinsumBuilder("ij,jk->ik", [(16, 32), (32, 16)], torch.float32)
    b.parse_equation()
    b.generate_code()
    b.compile()
    tagged = re.search(r"einsum_[0-9a-f]{32}_[0-9a-f]{8}\.so$", b.so_filename)
    assert bool(tagged) == (stop is not None)
    syms = _undefined_symbols(b.so_filename)
    gated = stop is not None and stop < 3
    assert ("pe_contract_ws_phase" in syms) == gated
    assert ("pe_contract_ws" in syms) == (not gated)
    b.cleanup()


def test_compile_failure_is_loud(monkeypatch):
    b = EinsumBuilder("ij,jk->ik", [(16, 32), (32, 16)], torch.float32)
    b.parse_equation()
    b.generate_code()
    b.cpp_code += "\n#error injected\n"
    b.code_hash = "0" * 32
    b.target_dir = os.path.join(b.build_base, b.code_hash)
    with pytest.raises(RuntimeError, match="Compilation failed"):
        b.compile()
    b.cleanup()
