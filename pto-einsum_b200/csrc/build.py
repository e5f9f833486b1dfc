"""Build libpto_einsum_b200.so (all CUDA sources, sm_100a) into pto_einsum/_lib/.

Usage: python build.py [--force]
The library is rebuilt when any source under csrc/ or include/ is newer than it.
"""
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(HERE), "pto_einsum")
REPO = os.path.dirname(os.path.dirname(HERE))
INCLUDE = os.path.join(REPO, "include")
OUT_DIR = os.path.join(PKG, "_lib")
OUT = os.path.join(OUT_DIR, "libpto_einsum_b200.so")
SOURCES = ["pe_api.cu", "pe_stream.cu", "pe_permute.cu", "pe_gemm.cu", "pe_noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _inputs():
    files = [os.path.join(HERE, f) for f in sorted(os.listdir(HERE))
             if f.endswith((".cu", ".cuh", ".h"))]
    files += [os.path.join(INCLUDE, f) for f in sorted(os.listdir(INCLUDE)) if f.endswith(".h")]
    return files


def source_hash() -> str:
    h = hashlib.md5()
    for f in _inputs():
        with open(f, "rb") as fh:
            h.update(os.path.basename(f).encode())
            h.update(fh.read())
    return h.hexdigest()[:12]


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(f) > t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile each source to an object in parallel, then link the library."""
    if not force and not needs_build():
        return OUT
    import tempfile
    from concurrent.futures import ThreadPoolExecutor
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    tag = source_hash()
    tmp = OUT + ".tmp"
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
             "-I", INCLUDE, "-I", HERE, f'-DPE_BUILD_TAG="{tag}"']
    if verbose:
        flags.append("-Xptxas=-v")
    with tempfile.TemporaryDirectory(prefix="pe_build_") as td:
        objs = [os.path.join(td, s.replace(".cu", ".o")) for s in SOURCES]

        def one(k):
            return subprocess.run([nvcc, *flags, "-c", os.path.join(HERE, SOURCES[k]), "-o", objs[k]],
                                  capture_output=True, text=True)
        with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
            results = list(ex.map(one, range(len(SOURCES))))
        for r in results:
            if r.returncode != 0:
                raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
            if verbose:
                sys.stderr.write(r.stderr)
        r = subprocess.run([nvcc, *ARCH, "-shared", *objs, "-o", tmp], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc link failed:\n" + r.stdout + r.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
