#!/usr/bin/env python
"""Benchmark of the B200 einsum hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl ours|reference]

A step is one einsum call (one fused launch on the contraction routes) over
one full BASELINE config, inputs resident in HBM. Under torchrun each rank
runs its own full-size shard of the batch axis (weak scaling: global batch =
N x config batch); there is no collective on the data path. Timing: CUDA
events on the launching stream around exactly K steps, bracketed by a
barrier and torch.cuda.synchronize(), max over ranks.

Default config is BASELINE config 2 ('bij,bjk->bik' fp16 -> fp32, b=64,
i=j=k=1024), the contraction the metric is quoted on; --config selects the
others (names in tests/corpus.py CONFIGS). Inputs are synthetic, seeded.

--impl reference times the reference's own CPU implementation (the libraries
oracle/build_ref.py compiled from the reference sources, oracle/_ref) on all
host threads, on bounded slices of the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "pto-einsum_b200"))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "tests"))

import torch  # noqa: E402

from corpus import CONFIGS  # noqa: E402

CFG = {name: (eq, s0, s1, dt) for name, eq, s0, s1, dt in CONFIGS}

# per config: (metric kind, bound, unit of work per call)
#   flops = 2*I*L0*L1*C; bytes = inputs read once + fp32 output written once
def work(name):
    eq, s0, s1, dt = CFG[name]
    from pto_einsum import planner
    r, _ = planner.choose_operand_order("cuda", eq, s0, s1)
    es = 2 if dt == "float16" else 4
    n0, n1 = 1, 1
    for d in s0:
        n0 *= d
    for d in s1:
        n1 *= d
    nbytes = es * (n0 + n1) + 4 * r["n_elem"]
    if r["elementwise"] or r["broadcast"]:
        return dict(kind="bytes", bound="hbm", flops=0, bytes=nbytes, recipe=r)
    flops = 2 * r["I"] * r["L0"] * r["L1"] * r["C"]
    # Contractions report TFLOP/s (BASELINE metric). The binding roof is the
    # larger of the two floors: tensor time at the measured peak (fp32 via
    # 3xTF32: three tf32 MMAs per product at half the bf16 rate, so an
    # effective peak of bf16 / 6) and HBM time for the algorithmic bytes.
    hbm, tflops, _ = peaks()
    tensor_peak = tflops / (6.0 if es == 4 else 1.0)
    t_tensor = flops / (tensor_peak * 1e12)
    t_hbm = nbytes / (hbm * 1e9)
    bound = "tensor" if t_tensor >= 0.9 * t_hbm else "hbm"
    return dict(kind="flops", bound=bound, flops=flops, bytes=nbytes, recipe=r, tensor_peak=tensor_peak)


def metric_of(w):
    if w["kind"] == "flops":
        return "einsum TFLOP/s", "TFLOP/s"
    return "einsum HBM GB/s", "GB/s"


def make_inputs(name, device, rank):
    eq, s0, s1, dt = CFG[name]
    dtype = getattr(torch, dt)
    g = torch.Generator(device="cpu").manual_seed(1000 + rank)
    if name in ("cfg2",):
        a = torch.rand(s0, generator=g, dtype=torch.float32)
        b = torch.rand(s1, generator=g, dtype=torch.float32)
    elif name == "cfg4b":
        a = torch.randn(s0, generator=g, dtype=torch.float32)
        t = torch.arange(s0[0], dtype=torch.float32)
        diff = t[:, None] - t[None, :]
        b = torch.where(diff >= 0, torch.pow(torch.tensor(0.99), diff.clamp(min=0)), torch.zeros(()))
    elif name == "cfg5_rms":
        a = torch.randn(s0, generator=g)
        b = torch.rand(s1, generator=g) + 0.5
    elif name == "cfg5_rope":
        a = torch.randn(s0, generator=g)
        S, D = s1
        pos = torch.arange(S, dtype=torch.float64)[:, None]
        j = torch.arange(D // 2, dtype=torch.float64)[None, :]
        ang = pos * torch.pow(10000.0, -2.0 * j / D)
        b = torch.cat([torch.cos(ang), torch.sin(ang)], dim=1).float()
    elif name == "cfg5_alibi":
        a = torch.randn(s0, generator=g)
        H = s1[0]
        b = torch.pow(2.0, -8.0 * (torch.arange(H, dtype=torch.float64) + 1) / H).float()
    else:
        a = torch.randn(s0, generator=g)
        b = torch.randn(s1, generator=g)
    return a.to(dtype).to(device), b.to(dtype).to(device)


class Clocks:
    """Sample nvidia-smi clocks / throttle reasons while the benchmark runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t0, t1):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ts, line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            rows.append((ts, f))
        inside = [r for r in rows if t0 - 0.05 <= r[0] <= t1 + 0.05] or rows
        sm = [float(f[1]) for _, f in inside if f[1].replace(".", "").isdigit()]
        mx = [float(f[2]) for _, f in inside if f[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for _, f in inside for k in range(4) if f[5 + k] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside)}


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def traffic_of(name):
    p = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(name)
    return None


def cpu_reference(name, seconds_budget=None, threads=None):
    """Time the reference's compiled CPU library on slices of `name`.
    Returns (units per second in the config's metric unit, cores, sample text)."""
    from oracle import ref_cpu
    if not ref_cpu.available():
        return None
    spec_name = next((n for n in ref_cpu.names() if ref_cpu.spec(n)["config"] == name), None)
    if spec_name is None:
        return None
    s = ref_cpu.spec(spec_name)
    threads = threads or min(os.cpu_count() or 1, 32)
    a, b = ref_cpu.sample_inputs(spec_name, seed=0)
    ref_cpu.run(spec_name, a, b)  # warm (loads the library, page-faults the output)
    outs = [None] * threads

    def worker(k):
        outs[k] = ref_cpu.run(spec_name, a, b, outs[k])

    t0 = time.perf_counter()
    ths = [threading.Thread(target=worker, args=(k,)) for k in range(threads)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    dt = time.perf_counter() - t0
    w = work(name)
    frac = 1.0 / s["units"]
    per_slice = (w["flops"] if w["kind"] == "flops" else w["bytes"]) * frac
    rate = per_slice * threads / dt / (1e12 if w["kind"] == "flops" else 1e9)
    sample = (f"{threads} concurrent calls of the reference CPU library for slice {spec_name} "
              f"({s['equation']} {tuple(s['shape0'])}x{tuple(s['shape1'])}, 1/{s['units']} of {name}), "
              f"{dt:.2f} s wall")
    return rate, threads, sample, dt


def run_reference_arm(args, rank, world):
    name = args.config
    w = work(name)
    metric, unit = metric_of(w)
    if rank != 0:
        return
    from oracle import ref_cpu
    if not ref_cpu.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (reference CPU libraries) not built"}))
        return
    threads = min(os.cpu_count() or 1, 32)
    for _ in range(args.warmup):
        cpu_reference(name, threads=threads)
    vals, times = [], []
    sample = None
    for _ in range(args.steps):
        rate, cores, sample, dt = cpu_reference(name, threads=threads)
        vals.append(rate)
        times.append(dt)
    value = statistics.median(vals)
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": name, "equation": CFG[name][0], "shape0": CFG[name][1],
                       "shape1": CFG[name][2], "input_dtype": CFG[name][3]},
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def _time(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_callers_suite(args):
    """Chained callers: the reference's LLM contraction patterns and the
    linear-attention chain (bench_linear_attention.py), B200 vs torch.einsum."""
    from llm_patterns import LARGE, PATTERNS, shapes
    from pto_einsum import EinsumBuilder
    from oracle.oracle import rel_frobenius
    dev = torch.device("cuda", 0)
    steps, warmup = max(args.steps // 10, 5), args.warmup
    for dt in (torch.float16, torch.float32):
        for name, eq in PATTERNS:
            s0, s1 = shapes(eq, LARGE)
            g = torch.Generator(device="cpu").manual_seed(7)
            a = torch.randn(s0, generator=g).to(dt).to(dev)
            b = torch.randn(s1, generator=g).to(dt).to(dev)
            run = EinsumBuilder(eq, [s0, s1], dt).build()
            ms = _time(lambda: run(a, b), steps, warmup)
            mt = _time(lambda: torch.einsum(eq, a, b), steps, warmup)
            err = rel_frobenius(run(a, b).cpu().numpy(), torch.einsum(eq, a.float(), b.float()).cpu().numpy())
            print(json.dumps({"suite": "callers", "op": name, "equation": eq, "dtype": str(dt).split(".")[-1],
                              "shape0": s0, "shape1": s1, "ms": round(ms, 4), "torch_ms": round(mt, 4),
                              "speedup_vs_torch": round(mt / ms, 3), "rel_frobenius_vs_torch_fp32": err}))
            del a, b, run
            torch.cuda.empty_cache()
        # linear-attention chain tn,sn,sp,ts->tp as three two-way einsums (config 4)
        T, N, P = 8192, 128, 128
        g = torch.Generator(device="cpu").manual_seed(8)
        Q = torch.randn(T, N, generator=g).to(dt).to(dev)
        K = torch.randn(T, N, generator=g).to(dt).to(dev)
        V = torch.randn(T, P, generator=g).to(dt).to(dev)
        t = torch.arange(T, dtype=torch.float32, device=dev)
        D = torch.where(t[:, None] >= t[None, :], torch.pow(0.99, (t[:, None] - t[None, :]).clamp(min=0)),
                        torch.zeros((), device=dev)).to(dt)
        r1 = EinsumBuilder("tn,sn->ts", [(T, N), (T, N)], dt).build()
        r2 = EinsumBuilder("ts,ts->ts", [(T, T), (T, T)], dt).build()
        r3 = EinsumBuilder("ts,sp->tp", [(T, T), (T, P)], dt).build()
        chain = lambda: r3(r2(r1(Q, K).to(dt), D).to(dt), V)  # noqa: E731
        ms = _time(chain, steps, warmup)
        mt = _time(lambda: torch.einsum("tn,sn,sp,ts->tp", Q, K, V, D), steps, warmup)
        err = rel_frobenius(chain().cpu().numpy(),
                            torch.einsum("tn,sn,sp,ts->tp", Q.float(), K.float(), V.float(), D.float()).cpu().numpy())
        print(json.dumps({"suite": "callers", "op": "linear_attention_chain", "equation": "tn,sn,sp,ts->tp",
                          "dtype": str(dt).split(".")[-1], "T": T, "ms": round(ms, 4), "torch_ms": round(mt, 4),
                          "speedup_vs_torch": round(mt / ms, 3), "rel_frobenius_vs_torch_fp32": err}))


def run_permute_suite(args):
    """Transpose family (reference include/pto_einsum_transpose.h, benchmarks/base/
    bench_transpose.py): pe_permute on large N-D permutes, GB/s (read + write) vs the
    measured copy roof and vs torch's permute().contiguous(); plus the reference's
    transposing einsum 'ai,ja->ij' at a large size."""
    import ctypes
    from pto_einsum import EinsumBuilder, _core
    lib = _core.core_lib()

    class Plan(ctypes.Structure):
        _fields_ = [("dtype", ctypes.c_int32), ("dims", ctypes.c_int32),
                    ("from_shape", ctypes.c_int64 * 8), ("perm", ctypes.c_int32 * 8)]
    dev = torch.device("cuda", 0)
    hbm, _, _ = peaks()
    steps, warmup = max(args.steps // 10, 10), args.warmup
    cases = [((16, 4096, 32, 128), (0, 2, 1, 3)), ((8192, 8192), (1, 0)), ((64, 1024, 1024), (0, 2, 1)),
             ((16, 4096, 32, 128), (0, 2, 3, 1)), ((8, 2048, 32, 128), (3, 1, 0, 2))]
    for dt in (torch.float16, torch.float32):
        for shape, perm in cases:
            x = torch.randn(shape, device=dev).to(dt)
            out = torch.empty([shape[i] for i in perm], device=dev, dtype=dt)
            pl = Plan()
            pl.dtype = 0 if dt == torch.float32 else 1
            pl.dims = len(shape)
            for i, (d, q) in enumerate(zip(shape, perm)):
                pl.from_shape[i] = d
                pl.perm[i] = q
            st = torch.cuda.current_stream(dev).cuda_stream

            def ours():
                rc = lib.pe_permute(ctypes.byref(pl), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                    ctypes.c_void_p(st))
                assert rc == 0
            ms = _time(ours, steps, warmup)
            mt = _time(lambda: x.permute(perm).contiguous(), steps, warmup)
            ok = torch.equal(out, x.permute(perm).contiguous())
            nbytes = 2 * x.numel() * x.element_size()
            print(json.dumps({"suite": "permute", "shape": shape, "perm": perm, "dtype": str(dt).split(".")[-1],
                              "ms": round(ms, 4), "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                              "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 3),
                              "torch_GB/s": round(nbytes / (mt * 1e-3) / 1e9, 1), "exact": ok}))
        n = 8192
        a = torch.rand(n, n, device=dev).to(dt)
        b = torch.rand(n, n, device=dev).to(dt)
        run = EinsumBuilder("ai, ja -> ij", [(n, n), (n, n)], dt).build()
        ms = _time(lambda: run(a, b), max(steps // 4, 3), warmup)
        mt = _time(lambda: torch.einsum("ai,ja->ij", a, b), max(steps // 4, 3), warmup)
        print(json.dumps({"suite": "permute", "op": "einsum ai,ja->ij (transposed operands)", "n": n,
                          "dtype": str(dt).split(".")[-1], "ms": round(ms, 4), "TFLOP/s": round(2 * n**3 / (ms * 1e-3) / 1e12, 1),
                          "torch_ms": round(mt, 4)}))


def run_thin_suite(args):
    """Thin outputs and few-tile long contractions: dot and matrix-vector products
    (streaming thin-output kernel) and thin GEMMs (stream-K), each vs torch.einsum,
    with the relative Frobenius error against float64. For the GEMM cases the same
    call with stream-K disabled (PE_GEMM_STREAMK=0, split-K only) is timed too."""
    from pto_einsum import EinsumBuilder
    dev = torch.device("cuda", 0)
    steps = max(args.steps // 10, 10)
    cases = [("i, i ->", (1 << 26,), (1 << 26,)), ("ij, j -> i", (256, 1 << 18), (1 << 18,)),
             ("bhd, bhd -> bh", (16, 32, 1 << 14), (16, 32, 1 << 14)),
             ("ij, jk -> ik", (128, 1 << 20), (1 << 20, 128)), ("ts, sp -> tp", (8192, 8192), (8192, 128))]
    for dt in (torch.float32, torch.float16):
        for eq, s0, s1 in cases:
            g = torch.Generator(device=dev).manual_seed(7)
            a = torch.randn(s0, device=dev, generator=g).to(dt)
            b = torch.randn(s1, device=dev, generator=g).to(dt)
            exact = torch.einsum(eq, a.double(), b.double())
            row = {"suite": "thin", "equation": eq, "shape0": list(s0), "shape1": list(s1),
                   "dtype": str(dt).split(".")[-1]}
            nbytes = (a.numel() + b.numel()) * a.element_size()
            modes = [("", None)] + ([("splitk_", "0")] if "k" in eq.split("->")[0] else [])
            for tag, env in modes:
                old = os.environ.get("PE_GEMM_STREAMK")
                if env is not None:
                    os.environ["PE_GEMM_STREAMK"] = env
                try:
                    bld = EinsumBuilder(eq, [s0, s1], dt)
                    run = bld.build()
                    ms = _time(lambda: run(a, b), steps, 3)
                    out = run(a, b).double()
                    bld.cleanup()
                finally:
                    if env is not None:
                        if old is None:
                            os.environ.pop("PE_GEMM_STREAMK", None)
                        else:
                            os.environ["PE_GEMM_STREAMK"] = old
                row[f"{tag}us"] = round(ms * 1e3, 1)
                row[f"{tag}rel_err"] = float(((out - exact).norm() / exact.norm()).item())
            row["input_GB/s"] = round(nbytes / (row["us"] * 1e-6) / 1e9, 1)
            row["torch_us"] = round(_time(lambda: torch.einsum(eq, a, b), steps, 3) * 1e3, 1)
            print(json.dumps(row), flush=True)


# The reference's base benchmark families (benchmarks/base/bench_einsum.py:32-178):
# (key, equation, dtype, sizes, shapes(size)), and its transposing einsum cases
# (benchmarks/base/bench_transpose.py:14-18).
BASE_FAMILIES = [
    ("matmul", "ij, jk -> ik", "float32", [128, 256, 512, 1024, 2048], lambda n: ((n, n), (n, n))),
    ("matmul-fp16", "ij, jk -> ik", "float16", [128, 256, 512, 1024, 2048], lambda n: ((n, n), (n, n))),
    ("transpose", "ji, jk -> ik", "float32", [128, 256, 512, 1024], lambda n: ((2 * n, n), (2 * n, n))),
    ("outer", "i, j -> ij", "float32", [256, 512, 1024, 2048], lambda n: ((n,), (n,))),
    ("dot-product", "i, i -> ", "float32", [4096, 16384, 49152, 131072], lambda n: ((n,), (n,))),
    ("batch-matmul", "bij, bjk -> bik", "float32", [8, 16, 32, 64, 128], lambda b: ((b, 64, 128), (b, 128, 64))),
    ("batch-matmul-tiny", "bij, bjk -> bik", "float32", [16, 32, 64, 128, 256],
     lambda b: ((b, 128, 128), (b, 128, 128))),
    ("batch-matmul-tiny-fp16", "bij, bjk -> bik", "float16", [16, 32, 64, 128, 256],
     lambda b: ((b, 128, 128), (b, 128, 128))),
    ("contraction", "ijk, jkl -> il", "float32", [32, 64, 128, 256], lambda k: ((64, 64, k), (64, k, 64))),
    ("custom-layout", "abc, cd -> abd", "float32", [8, 16, 32, 64], lambda a: ((a, 64, 128), (128, 256))),
    ("gdn-kkt-nt", "bihd, bjhd -> bihj", "float32", [8, 16, 32, 64],
     lambda b: ((b, 128, 16, 128), (b, 128, 16, 128))),
    ("gdn-wy-fast-nn", "bihj, bjhd -> bihd", "float32", [8, 16, 32, 64],
     lambda b: ((b, 128, 16, 128), (b, 128, 16, 128))),
    ("gdn-chunk-h-tn", "bvhd, bvhe -> bhde", "float32", [8, 16, 32, 64],
     lambda b: ((b, 128, 16, 128), (b, 128, 16, 128))),
    ("unaligned", "ij, jk -> ik", "float32", [128, 256, 512, 1024], lambda n: ((n, n - 6), (n - 6, n))),
    ("batch-unaligned", "bij, bjk -> bik", "float32", [8, 16, 32, 64], lambda b: ((b, 64, 100), (b, 100, 64))),
    ("transpose-2d", "ai, ja -> ij", "float32", [64, 256, 512], lambda n: ((n, n), (n, n))),
]


def run_base_suite(args):
    """The reference's base benchmark sweep on one B200: per point the build time,
    the median host wall time of one call followed by a synchronize (the reference's
    own method, bench_einsum.py:183-215) for this library and torch.einsum, the
    device time per call of back-to-back calls (CUDA events), and the relative
    Frobenius error against float64. Inputs U[0,1) as in the reference."""
    from pto_einsum import EinsumBuilder
    dev = torch.device("cuda", 0)
    runs = max(args.steps // 2, 20)
    for key, eq, dts, sizes, make in BASE_FAMILIES:
        dt = getattr(torch, dts)
        for n in sizes:
            s0, s1 = make(n)
            a = torch.rand(s0, device=dev).to(dt)
            b = torch.rand(s1, device=dev).to(dt)
            row = {"suite": "base", "family": key, "equation": eq, "dtype": dts, "size": n,
                   "shape0": list(s0), "shape1": list(s1)}
            t0 = time.perf_counter()
            try:
                bld = EinsumBuilder(eq, [s0, s1], dt)
                run = bld.build()
            except ValueError as e:
                row["unsupported"] = str(e)[:120]
                print(json.dumps(row))
                continue
            row["build_s"] = round(time.perf_counter() - t0, 3)

            def wall(fn):
                for _ in range(5):
                    fn()
                torch.cuda.synchronize()
                ts = []
                for _ in range(runs):
                    t = time.perf_counter()
                    fn()
                    torch.cuda.synchronize()
                    ts.append((time.perf_counter() - t) * 1e3)
                return statistics.median(ts)
            ours = lambda: run(a, b)  # noqa: E731
            theirs = lambda: torch.einsum(eq, a, b)  # noqa: E731
            row["ms"] = round(wall(ours), 4)
            row["torch_ms"] = round(wall(theirs), 4)
            row["speedup"] = round(row["torch_ms"] / row["ms"], 3)
            row["device_us"] = round(_time(ours, runs, 3) * 1e3, 2)
            row["torch_device_us"] = round(_time(theirs, runs, 3) * 1e3, 2)
            exact = torch.einsum(eq, a.double(), b.double())
            got = run(a, b).double()
            den = exact.norm().item()
            row["rel_err"] = float(((got - exact).norm() / den).item()) if den else 0.0
            bld.cleanup()
            print(json.dumps(row), flush=True)


def run_gdn_suite(args):
    """GDN stage backends (the reference's benchmarks/complex/gdn/bench_gdn_4way.py
    workloads: N_seq x L_seg in {1,2} x {512,1024}, H=32 value heads, Hg=16 key heads,
    head dim 128, chunk 128, fp32). Per stage: median device time with a 256 MB L2
    flush before each sample, torch.einsum backend vs this library's kernels on the
    same glue; then the whole forward eager and as one CUDA graph. Error = relative
    Frobenius vs the same pipeline in float64 (torch)."""
    from pto_einsum.gdn import GDNChunked, GDNGraph, random_gdn_inputs
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    iters = max(args.steps // 10, 10)

    def med(fn, warmup=3):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    def rel(a, b):
        a, b = a.double(), b.double()
        return ((a - b).norm() / b.norm()).item()

    H, Hg, D, C = 32, 16, 128, 128
    for n_seq, l_seg in [(1, 512), (2, 512), (1, 1024), (2, 1024)]:
        T = n_seq * l_seg
        cu = list(range(0, T + 1, l_seg))
        q, k, v, g, beta = random_gdn_inputs(T, H, Hg, D, seed=T + n_seq, device=dev)
        scale = D ** -0.5
        row = {"suite": "gdn", "N_seq": n_seq, "L_seg": l_seg, "T": T, "H": H, "Hg": Hg, "D": D, "chunk": C,
               "dtype": "float32"}
        ref = GDNChunked("torch", chunk=C, dtype=torch.float64)(
            *(x.double() for x in (q, k, v, g, beta)), scale=scale, cu_seqlens=cu)
        for name in ("torch", "pto"):
            m = GDNChunked(name, chunk=C)
            f = lambda x: m.fold(x, cu)  # noqa: E731
            qf, kf, vf, gf, bf = f(q), f(k), f(v), f(g), f(beta)
            gcum = m.cumsum(gf)
            A = m.kkt(kf, bf, gcum)
            Ainv = m.solve_tril(A)
            w, u = m.wy_fast(kf, vf, bf, Ainv, gcum)
            h, vn, _ = m.chunk_h(kf, w, u, gcum)
            stages = {
                "kkt": lambda: m.kkt(kf, bf, gcum),
                "solve_tril": lambda: m.solve_tril(A),
                "wy_fast": lambda: m.wy_fast(kf, vf, bf, Ainv, gcum),
                "chunk_h": lambda: m.chunk_h(kf, w, u, gcum),
                "chunk_o": lambda: m.chunk_o(qf, kf, vn, h, gcum),
            }
            row[f"{name}_stage_ms"] = {st: round(med(fn), 4) for st, fn in stages.items()}
            row[f"{name}_contraction_stages_ms"] = round(sum(v for st, v in row[f"{name}_stage_ms"].items()
                                                             if st != "solve_tril"), 4)
            row[f"{name}_forward_ms"] = round(med(lambda: m(q, k, v, g, beta, scale=scale, cu_seqlens=cu)), 4)
            graph = GDNGraph(m, q, k, v, g, beta, scale=scale, cu_seqlens=cu)
            row[f"{name}_forward_graph_ms"] = round(med(lambda: graph(q, k, v, g, beta)), 4)
            row[f"{name}_rel_err_vs_fp64"] = rel(m(q, k, v, g, beta, scale=scale, cu_seqlens=cu), ref)
            del graph
            if name == "pto":
                m.cleanup()
        print(json.dumps(row))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2", choices=sorted(CFG))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=16,
                    help="pipelined end-to-end steps (fill and drain cost about one step)")
    ap.add_argument("--suite", default=None, choices=["callers", "permute", "gdn", "base", "thin"],
                    help="instead of the one-line benchmark: time the LLM contraction patterns and the "
                         "linear-attention chain against torch.einsum (one JSON line per op)")
    ap.add_argument("--shrink", type=int, default=1,
                    help="divide the config's leading axis (small cases for profiler captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.shrink > 1:
        eq, s0, s1, dt = CFG[args.config]
        a0, b0 = eq.split("->")[0].split(",")
        lead = eq.split("->")[1][0]
        s0 = tuple(d // args.shrink if a0[i] == lead else d for i, d in enumerate(s0))
        s1 = tuple(d // args.shrink if b0[i] == lead else d for i, d in enumerate(s1))
        CFG[args.config] = (eq, s0, s1, dt)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.suite == "callers":
        run_callers_suite(args)
        return
    if args.suite == "permute":
        run_permute_suite(args)
        return
    if args.suite == "gdn":
        run_gdn_suite(args)
        return
    if args.suite == "base":
        run_base_suite(args)
        return
    if args.suite == "thin":
        run_thin_suite(args)
        return

    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    from pto_einsum import EinsumBuilder, _core
    name = args.config
    eq, s0, s1, dt = CFG[name]
    dtype = getattr(torch, dt)
    w = work(name)
    metric, unit = metric_of(w)
    a, b = make_inputs(name, device, rank)
    builder = EinsumBuilder(eq, [s0, s1], dtype, device=device)
    run = builder.build()
    stream = torch.cuda.current_stream(device)

    for _ in range(args.warmup):
        out = run(a, b)
    torch.cuda.synchronize(device)
    del out

    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.2)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    launches0 = _core.launch_count()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t_wall0 = time.time()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for k in range(args.steps):
        evs[k][0].record(stream)
        out = run(a, b)
        evs[k][1].record(stream)
    stop.record(stream)
    torch.cuda.synchronize(device)
    t_wall1 = time.time()
    if dist:
        dist.barrier()
    launches = _core.launch_count() - launches0
    elapsed_ms = start.elapsed_time(stop)
    per_launch_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
    clk = clocks.stop(t_wall0, t_wall1)
    if dist:
        t = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    assert _core.device_error(stream.cuda_stream) == 0, "device error word set"

    units_per_step = w["flops"] if w["kind"] == "flops" else w["bytes"]
    scale = 1e12 if w["kind"] == "flops" else 1e9
    value = units_per_step * args.steps * world / (elapsed_ms * 1e-3) / scale

    # ---- end to end through the public API with host buffers ----
    a_h = a.cpu().pin_memory()
    b_h = b.cpu().pin_memory()
    out_h = torch.empty(w["recipe"]["out_shape"], dtype=torch.float32).pin_memory()
    del out
    torch.cuda.synchronize(device)
    # Pipelined the way a streaming caller would: H2D of step k+1 and D2H of
    # step k-1 run on their own streams while step k computes (PCIe is full
    # duplex); device inputs are double-buffered. Every step still copies its
    # inputs in and its result out inside the timed region.
    e_steps = max(2, args.e2e_steps)
    s_h2d, s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ad = [torch.empty_like(a), torch.empty_like(a)]
    bd = [torch.empty_like(b), torch.empty_like(b)]
    h2d_done = [torch.cuda.Event(), torch.cuda.Event()]
    comp_done = [torch.cuda.Event(), torch.cuda.Event()]

    def e2e_step(k):
        j = k % 2
        if k >= 2:
            s_h2d.wait_event(comp_done[j])   # buffer j free once step k-2 computed
        with torch.cuda.stream(s_h2d):
            ad[j].copy_(a_h, non_blocking=True)
            bd[j].copy_(b_h, non_blocking=True)
            h2d_done[j].record(s_h2d)
        stream.wait_event(h2d_done[j])
        with torch.cuda.stream(stream):
            o = run(ad[j], bd[j])
            comp_done[j].record(stream)
        s_d2h.wait_event(comp_done[j])
        with torch.cuda.stream(s_d2h):
            out_h.copy_(o, non_blocking=True)
            o.record_stream(s_d2h)

    e2e_step(0)  # warm-up
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e0.record(s_h2d)
    for k in range(e_steps):
        e2e_step(k)
    e1 = torch.cuda.Event(enable_timing=True)
    s_d2h.wait_stream(stream)
    e1.record(s_d2h)
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = units_per_step * e_steps * world / (e2e_ms * 1e-3) / scale

    hbm, tflops, peak_src = peaks()
    if w["bound"] == "tensor":
        achieved = w["flops"] / (per_launch_ms * 1e-3) / 1e12
        peak = w.get("tensor_peak", tflops)
        if peak != tflops:
            peak_src += " (fp32 3xTF32: bf16 peak / 6)"
    else:
        achieved = w["bytes"] / (per_launch_ms * 1e-3) / 1e9
        peak = hbm
    traffic = traffic_of(name)

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            r = cpu_reference(name)
            if r:
                cpu = {"value": r[0], "unit": unit, "cores": r[1], "kind": "reference", "sample": r[2]}
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16" if dt == "float16" else "f32",
            "data": "synthetic (seeded)",
            "config": {"workload": name, "equation": eq, "shape0": s0, "shape1": s1, "input_dtype": dt,
                       "output_dtype": "float32", "global_batch": s0[0] * world,
                       "parallelism": f"batch-sharded x{world}, no collective",
                       "l2": "inputs+output larger than L2 (126 MB)"},
            "roofline": {"bound": w["bound"], "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s" if w["bound"] == "tensor" else "GB/s",
                         "frac": achieved / peak, "peak_source": peak_src, "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": unit,
                    "h2d_bytes_per_step": a.numel() * a.element_size() + b.numel() * b.element_size(),
                    "d2h_bytes_per_step": out_h.numel() * 4},
            "gpu_launches": launches,
            "clocks": clk,
        }
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
