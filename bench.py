#!/usr/bin/env python
"""Benchmark of the B200 einsum hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--configs all|none|a,b]
                    [--impl ours|reference] [--suite callers|permute|gdn|base|thin]

A step is one einsum call (one fused launch on the contraction routes) through
the public EinsumBuilder runner over one BASELINE config, inputs resident in
HBM. Under torchrun the config's leading output axis is split over the ranks
with the product's shard plan (pto_einsum.distributed): strong scaling, the
job does the config's work once, with no collective on the data path; the
weak-scaling figure (every rank the whole config) and the optional NCCL
all-gather of the result are reported beside it. Timing: CUDA events on the
launching stream around exactly K steps, bracketed by a barrier and
torch.cuda.synchronize(), max over ranks.

The headline is BASELINE config 2 ('bij,bjk->bik' fp16 -> fp32, b=64,
i=j=k=1024), the contraction the metric is quoted on; every other config
(names in tests/corpus.py CONFIGS) is measured into the line's `configs` map
with its own roofline, end-to-end figure, CPU baseline and sampled parity
against the CPU oracle. Inputs are synthetic, seeded, generated on the device.

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

import fullsize  # noqa: E402

CFG = fullsize.CFG   # name -> (equation, shape0, shape1, dtype name); --shrink edits it in place
L2_BYTES = 126 << 20

# per config: (metric kind, bound, unit of work per call)
#   flops = 2*I*L0*L1*C; bytes = inputs read once + fp32 output written once
def work(name, s0=None, s1=None):
    """Units of config `name` (or of its shard with shapes s0, s1) per call:
    flops = 2*I*L0*L1*C; bytes = inputs read once + fp32 output written once."""
    eq, f0, f1, dt = CFG[name]
    s0, s1 = tuple(s0 or f0), tuple(s1 or f1)
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
        return dict(kind="bytes", bound="hbm", flops=0, bytes=nbytes, recipe=r, units=nbytes)
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
    return dict(kind="flops", bound=bound, flops=flops, bytes=nbytes, recipe=r, tensor_peak=tensor_peak,
                units=flops)


def metric_of(w):
    if w["kind"] == "flops":
        return "einsum TFLOP/s", "TFLOP/s"
    return "einsum HBM GB/s", "GB/s"


class Clocks:
    """Sample the GPU's SM clock and throttle reasons in a background thread
    (NVML every 2 ms; nvidia-smi every 50 ms where NVML is unavailable), so
    even a timed region of a few milliseconds gets samples."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device):
        self.device = device
        self.samples = []          # (time, sm MHz, max MHz, set of reason names)
        self.proc = None
        self.nvml = None
        self.stop_flag = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.device)
        try:
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)

    def start(self):
        try:
            self.nvml = self._nvml_handle()
        except Exception:
            self.nvml = None
        if self.nvml:
            self.t = threading.Thread(target=self._poll_nvml, daemon=True)
            self.t.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device.index or 0}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read_smi, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None

    def _poll_nvml(self):
        nv, h = self.nvml
        bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self.stop_flag.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((time.time(), float(sm), float(mx),
                                     {n for n, b in zip(self.NAMES, bits) if r & b}))
            except Exception:
                pass
            time.sleep(0.002)

    def _read_smi(self):
        for line in self.proc.stdout:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[1].replace(".", "").isdigit():
                continue
            self.samples.append((time.time(), float(f[1]), float(f[2]) if f[2].replace(".", "").isdigit() else None,
                                 {self.NAMES[k] for k in range(4) if f[5 + k] == "Active"}))

    def summary(self, t0, t1):
        """Median SM clock, max clock and active throttle reasons of the samples
        taken in wall-clock window [t0, t1]."""
        if not self.nvml and self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        rows = list(self.samples)
        inside = [r for r in rows if t0 <= r[0] <= t1]
        if not inside:   # a window shorter than the sampling period: nearest sample
            inside = sorted(rows, key=lambda r: abs(r[0] - 0.5 * (t0 + t1)))[:1]
        sm = [r[1] for r in inside]
        mx = [r[2] for r in inside if r[2]]
        reasons = sorted(set().union(*[r[3] for r in inside])) if inside else []
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside), "source": "nvml" if self.nvml else "nvidia-smi"}

    def stop(self):
        self.stop_flag.set()
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()


def peaks(sustained=False):
    """(HBM GB/s, dense bf16 TFLOP/s, source): the driver-measured figures of
    MEASURED_PEAKS.json (burst GEMM rate, or the rate under the power cap with
    sustained=True), else this pool's earlier fallback measurement."""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        tf = d.get("bf16_tflops_sustained", 1376.6) if sustained else d.get("bf16_tflops", 1590.0)
        return d.get("hbm_gbs", 6650.0), tf, "measured" + (" (sustained)" if sustained else " (burst)")
    return 6650.0, (1400.0 if sustained else 1590.0), "fallback"


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
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
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


def run_host_suite(args):
    """Host cost per runner call: wall time per call of 200 calls submitted while
    the GPU is held busy by a sleep kernel (so only the host's submit cost is
    measured, never the GPU's rate), median of 7 samples; for the runner, the bare
    run_einsum_exec ctypes call, and torch.einsum. Run once more with
    PE_PLAN_CACHE=0 to see the cost without the prepared-launch cache."""
    import ctypes
    from pto_einsum import EinsumBuilder
    dev = torch.device("cuda", 0)
    cases = [("ij,jk->ik", (128, 128), (128, 128), torch.float32),
             ("ij,jk->ik", (128, 128), (128, 128), torch.float16),
             ("bij,bjk->bik", (8, 128, 128), (8, 128, 128), torch.float16),
             ("bshd,bthd->bsht", (1, 128, 4, 64), (1, 128, 4, 64), torch.float16),
             ("ts,ts->ts", (256, 256), (256, 256), torch.float32),
             ("bsd,d->bsd", (2, 64, 256), (256,), torch.float16)]

    def per_call_us(fn):
        # the GPU is held busy (torch.cuda._sleep) while the calls are timed, so
        # the wall time is the host's submit cost alone, never the GPU's rate
        for _ in range(50):
            fn()
        torch.cuda.synchronize()
        meds = []
        for _ in range(7):
            torch.cuda._sleep(200_000_000)
            t0 = time.perf_counter()
            for _ in range(200):
                fn()
            meds.append((time.perf_counter() - t0) / 200 * 1e6)
            torch.cuda.synchronize()
        return statistics.median(meds)

    for eq, s0, s1, dt in cases:
        a = torch.randn(s0, device=dev).to(dt)
        b = torch.randn(s1, device=dev).to(dt)
        bld = EinsumBuilder(eq, [s0, s1], dt)
        run = bld.build()
        row = {"suite": "host", "equation": eq, "shape0": s0, "shape1": s1, "dtype": str(dt).split(".")[-1],
               "cache": os.environ.get("PE_PLAN_CACHE", "1") != "0"}
        row["runner_us"] = round(per_call_us(lambda: run(a, b)), 2)
        out = run(a, b)
        ws = bld.workspace(dev, torch.cuda.current_stream().cuda_stream)
        st = torch.cuda.current_stream().cuda_stream
        ex = bld.lib.run_einsum_exec
        pa, pb, po = a.data_ptr(), b.data_ptr(), out.data_ptr()
        if bld._swap_operands:
            pa, pb = pb, pa
        row["exec_only_us"] = round(per_call_us(lambda: ex(pa, pb, po, ws, st)), 2)
        row["torch_einsum_us"] = round(per_call_us(lambda: torch.einsum(eq, a, b)), 2)
        print(json.dumps(row), flush=True)
        bld.cleanup()


def run_phases_suite(args):
    """The reference's phase-overlap study (benchmarks/profile_phase_overlap.py:72-128)
    on the fused kernel: each config built with EINSUM_PHASE_STOP = 0 (launch and
    pipeline barriers), 1 (+ operand loads), 2 (+ tensor-core MMAs), 3 (+ epilogue
    stores: the full kernel); CUDA-event time per call, the per-phase increments by
    subtraction. Contraction configs only (--configs selects)."""
    from pto_einsum import EinsumBuilder
    dev = torch.device("cuda", 0)
    names = [n for n in CFG if n not in ("cfg1",) and n not in fullsize.EXACT]
    if args.configs not in ("all", "none"):
        names = [n for n in args.configs.split(",") if n]
    steps = max(args.steps // 4, 20)
    for name in names:
        eq, s0, s1, dt = CFG[name]
        a, b = fullsize.make_inputs(name, device=dev)
        row = {"suite": "phases", "config": name, "equation": eq}
        for stop in (0, 1, 2, 3):
            os.environ["EINSUM_EXTRA_DEFINES"] = f"-DEINSUM_PHASE_STOP={stop}"
            bld = EinsumBuilder(eq, [s0, s1], getattr(torch, dt))
            run = bld.build()
            row[f"stop{stop}_us"] = round(_time(lambda: run(a, b), steps, 3) * 1e3, 2)
            bld.cleanup()
        os.environ.pop("EINSUM_EXTRA_DEFINES", None)
        row["barriers_us"] = row["stop0_us"]
        row["loads_us"] = round(row["stop1_us"] - row["stop0_us"], 2)
        row["mma_us"] = round(row["stop2_us"] - row["stop1_us"], 2)
        row["epilogue_us"] = round(row["stop3_us"] - row["stop2_us"], 2)
        print(json.dumps(row), flush=True)
        del a, b
        torch.cuda.empty_cache()


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


def run_kda_suite(args):
    """KDA stage backends (the reference's benchmarks/complex/kda/bench_kda_4way.py
    workloads: N_seq x L_seg in {1,2} x {512,1024}, H=32 value heads, Hk=16 key heads,
    head dim 128, chunk 128, fp32, per-dimension gate in (-0.05, 0]): per stage median
    device time with a 256 MB L2 flush before each sample, torch.einsum backend vs
    this library's kernels on the same glue, the whole forward eager and as one CUDA
    graph, and the relative Frobenius error against the same pipeline in float64."""
    from pto_einsum.kda import KDAChunked, KDAGraph, random_kda_inputs
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

    H, Hk, D, C = 32, 16, 128, 128
    for n_seq, l_seg in [(1, 512), (2, 512), (1, 1024), (2, 1024)]:
        T = n_seq * l_seg
        cu = list(range(0, T + 1, l_seg))
        q, k, v, g, beta = random_kda_inputs(T, H, Hk, D, seed=T + n_seq, device=dev)
        scale = D ** -0.5
        row = {"suite": "kda", "N_seq": n_seq, "L_seg": l_seg, "T": T, "H": H, "Hk": Hk, "D": D, "chunk": C,
               "dtype": "float32"}
        ref = KDAChunked("torch", chunk=C, dtype=torch.float64)(
            *(x.double() for x in (q, k, v, g, beta)), scale=scale, cu_seqlens=cu)
        for name in ("torch", "pto"):
            m = KDAChunked(name, chunk=C)
            f = lambda x: m.fold(x, cu)  # noqa: E731
            qf, kf, vf, gf, bf = f(q), f(k), f(v), f(g), f(beta)
            gcum = m.cumsum(gf)
            A = m.kkt(kf, bf, gcum)
            Ainv = m.solve_tril(A)
            w, u = m.wy_fast(kf, vf, bf, Ainv, gcum)
            h, vn, _ = m.chunk_h(kf, w, u, gcum)
            stages = {
                "kkt": lambda: m.kkt(kf, bf, gcum),
                "wy_fast": lambda: m.wy_fast(kf, vf, bf, Ainv, gcum),
                "chunk_h": lambda: m.chunk_h(kf, w, u, gcum),
                "chunk_o": lambda: m.chunk_o(qf, kf, vn, h, gcum),
            }
            row[f"{name}_stage_ms"] = {st: round(med(fn), 4) for st, fn in stages.items()}
            row[f"{name}_forward_ms"] = round(med(lambda: m(q, k, v, g, beta, scale=scale, cu_seqlens=cu)), 4)
            graph = KDAGraph(m, q, k, v, g, beta, scale=scale, cu_seqlens=cu)
            row[f"{name}_forward_graph_ms"] = round(med(lambda: graph(q, k, v, g, beta)), 4)
            row[f"{name}_rel_err_vs_fp64"] = rel(m(q, k, v, g, beta, scale=scale, cu_seqlens=cu), ref)
            del graph
            if name == "pto":
                m.cleanup()
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




def _max_over_ranks(x, dist, device):
    if not dist:
        return x
    t = torch.tensor([x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(dist, device):
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)


def measure(name, args, rank, world, dist, device, clocks, *, steps, shard=True, cpu=False, parity=True,
            e2e=True, sustained_ms=None):
    """Time config `name` through the public EinsumBuilder runner.

    shard=True: the config's leading output axis is split over the ranks with
    the product's shard plan (pto_einsum.distributed.shard_operands), so the
    job does the config's work once (strong scaling). shard=False: every rank
    runs the whole config (weak scaling). Inputs are generated on the device
    from seeded generators (the shards concatenate to the one-device inputs)."""
    from pto_einsum import EinsumBuilder, _core
    from pto_einsum.distributed import shard_operands
    t_start = time.time()
    sustained_ms = args.sustained_ms if sustained_ms is None else sustained_ms
    eq, _, _, dt = CFG[name]
    dtype = getattr(torch, dt)
    full = work(name)
    metric, unit = metric_of(full)
    a, b = fullsize.make_inputs(name, device=device)
    if shard and world > 1:
        a, b = shard_operands(eq, a, b, rank, world)
    ls0, ls1 = tuple(a.shape), tuple(b.shape)
    local = work(name, ls0, ls1)
    job_units = full["units"] if shard else full["units"] * world
    builder = EinsumBuilder(eq, [ls0, ls1], dtype, device=device)
    run = builder.build()
    stream = torch.cuda.current_stream(device)
    out_bytes = 4 * local["recipe"]["n_elem"]
    in_bytes = a.numel() * a.element_size() + b.numel() * b.element_size()
    # Consecutive steps must not find their data in L2: below twice the L2 size
    # the step rotates over several input sets (and keeps that many outputs
    # alive, so the allocator hands out distinct output blocks).
    foot = in_bytes + out_bytes
    nsets = 1 if foot >= 2 * L2_BYTES else min(16, -(-2 * L2_BYTES // foot))
    sets = [(a, b)] + [(a.clone(), b.clone()) for _ in range(nsets - 1)]
    l2_note = ("inputs+output larger than 2x L2 (126 MB)" if nsets == 1 else
               f"rotating {nsets} input/output sets of {foot / 1e6:.0f} MB ({nsets * foot / 1e6:.0f} MB > 2x L2)")
    outs = [None] * nsets
    for k in range(max(args.warmup, 3)):
        outs[k % nsets] = run(*sets[k % nsets])
    torch.cuda.synchronize(device)
    _barrier(dist, device)
    launches0 = _core.launch_count()
    # Only the two events that bracket the region: an event recorded between two
    # steps would sit between their launches and stop the next launch's prologue
    # from overlapping the previous one's tail (programmatic dependent launch),
    # which a caller running steps back to back gets.
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_win0 = time.time()
    start.record(stream)
    for k in range(steps):
        j = k % nsets
        outs[j] = run(*sets[j])
    stop.record(stream)
    torch.cuda.synchronize(device)
    t_win1 = time.time()
    launches = _core.launch_count() - launches0
    _barrier(dist, device)
    elapsed_ms = _max_over_ranks(start.elapsed_time(stop), dist, device)
    per_launch_ms = start.elapsed_time(stop) / steps  # this rank's mean step (one runner call)
    clk = clocks.summary(t_win0, t_win1)

    # Sustained: about one second of back-to-back steps, where the 1 kW power
    # cap settles the clocks; reported beside the K-step figure.
    per_step_ms = max(elapsed_ms / steps, 1e-3)
    n_sus = min(max(steps, int(sustained_ms / per_step_ms)), 20000) if sustained_ms > 0 else steps
    _barrier(dist, device)
    s0e, s1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_s0 = time.time()
    s0e.record(stream)
    for k in range(n_sus):
        j = k % nsets
        outs[j] = run(*sets[j])
    s1e.record(stream)
    torch.cuda.synchronize(device)
    t_s1 = time.time()
    sus_ms = _max_over_ranks(s0e.elapsed_time(s1e), dist, device)
    sus_clk = clocks.summary(t_s0 + 0.5 * (t_s1 - t_s0), t_s1)   # second half: settled
    assert _core.device_error(stream.cuda_stream) == 0, "device error word set"
    scale = 1e12 if full["kind"] == "flops" else 1e9
    value = job_units * steps / (elapsed_ms * 1e-3) / scale
    sus_value = job_units * n_sus / (sus_ms * 1e-3) / scale

    def roof(ms_per_launch, sustained):
        hbm, tflops, src = peaks(sustained)
        if full["bound"] == "tensor":
            ach = local["flops"] / (ms_per_launch * 1e-3) / 1e12
            pk = tflops / (6.0 if dt == "float32" else 1.0)
            if dt == "float32":
                src += " (fp32 3xTF32: bf16 peak / 6)"
        else:
            ach = local["bytes"] / (ms_per_launch * 1e-3) / 1e9
            pk = hbm
        return ach, pk, src

    achieved, peak, peak_src = roof(per_launch_ms, False)
    s_ach, s_peak, s_src = roof(sus_ms / n_sus, True)
    traffic = traffic_of(name)
    traffic_note = "ncu dram read+write bytes of one full-size launch"
    if traffic is not None and local["units"] != full["units"]:
        traffic = traffic * local["units"] / full["units"]
        traffic_note = "full-size launch's ncu dram bytes scaled by this rank's share of the work"
    res = {"metric": metric, "unit": unit, "value": value, "ms_per_step": elapsed_ms / steps, "steps": steps,
           "dtype": "f16" if dt == "float16" else "f32",
           "config": {"workload": name, "equation": eq, "shape0": list(CFG[name][1]),
                      "shape1": list(CFG[name][2]), "local_shape0": list(ls0), "local_shape1": list(ls1),
                      "input_dtype": dt, "output_dtype": "float32", "l2": l2_note},
           "roofline": {"bound": full["bound"], "achieved": achieved, "peak": peak,
                        "unit": "TFLOP/s" if full["bound"] == "tensor" else "GB/s",
                        "frac": achieved / peak, "peak_source": peak_src, "traffic": traffic,
                        "traffic_source": traffic_note, "per_launch_ms": per_launch_ms},
           "sustained": {"value": sus_value, "steps": n_sus, "ms_per_step": sus_ms / n_sus,
                         "roofline_frac": s_ach / s_peak, "peak": s_peak, "peak_source": s_src,
                         "clocks": sus_clk,
                         "how": "about 1 s of back-to-back steps after the timed region; clocks from its second half"},
           "gpu_launches": launches, "clocks": clk}

    if name == "cfg2" and shard:
        # the same contraction through cuBLAS (torch.bmm, fp16 in, fp32 out) on the
        # same inputs and stream: a library reference point, not a baseline arm
        try:
            bmm = lambda: torch.bmm(a, b, out_dtype=torch.float32)  # noqa: E731
            t_lib = _max_over_ranks(_time(bmm, steps, 3), dist, device)
            res["library_reference"] = {
                "what": "torch.bmm(a, b, out_dtype=torch.float32) (cuBLAS), same inputs, CUDA events",
                "value": job_units / (t_lib * 1e-3) / scale, "unit": unit, "ms_per_step": t_lib}
        except (TypeError, RuntimeError) as e:
            res["library_reference"] = {"unavailable": str(e)[:120]}
    if parity and rank == 0:
        out = run(a, b)
        chk = fullsize.check(name, a.cpu(), b.cpu(), out.cpu(), threads=min(os.cpu_count() or 1, 32),
                             whole_exact=False)
        chk["tolerance"] = 0.0 if name in fullsize.EXACT else fullsize.TOL[dt]
        chk["pass"] = chk["bit_exact"] if name in fullsize.EXACT else chk["rel_frobenius"] <= chk["tolerance"]
        chk["oracle"] = "oracle/einsum_oracle.c (restates the reference include/cpu_einsum.h:53-92)"
        res["parity"] = chk
        del out
    del outs, sets
    torch.cuda.empty_cache()

    if e2e:
        res["e2e"] = e2e_run(run, a, b, local, job_units, scale, unit, args, dist, device)
    if cpu and rank == 0 and world == 1:
        r = cpu_reference(name)
        if r:
            res["cpu_baseline"] = {"value": r[0], "unit": unit, "cores": r[1], "kind": "reference",
                                   "sample": r[2]}
    builder.cleanup()
    del a, b
    torch.cuda.empty_cache()
    res["wall_s"] = round(time.time() - t_start, 2)
    return res


def e2e_run(run, a, b, local, job_units, scale, unit, args, dist, device):
    """The same runner call end to end with host buffers: each step copies its
    inputs from pinned host memory and its result back inside the timed region.
    Pipelined the way a streaming caller runs it: host->device copies of step
    k+1 and device->host copies of step k-1 on their own streams while step k
    computes (PCIe is full duplex); device inputs double-buffered."""
    stream = torch.cuda.current_stream(device)
    a_h = a.cpu().pin_memory()
    b_h = b.cpu().pin_memory()
    out_h = torch.empty(local["recipe"]["out_shape"], dtype=torch.float32).pin_memory()
    step_bytes = a_h.numel() * a_h.element_size() + b_h.numel() * b_h.element_size() + out_h.numel() * 4
    e_steps = max(2, min(args.e2e_steps, int(8e9 // max(step_bytes, 1))))
    s_h2d, s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ad = [torch.empty_like(a), torch.empty_like(a)]
    bd = [torch.empty_like(b), torch.empty_like(b)]
    h2d_done = [torch.cuda.Event(), torch.cuda.Event()]
    comp_done = [torch.cuda.Event(), torch.cuda.Event()]

    def step(k):
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

    step(0)  # warm-up
    _barrier(dist, device)
    e0 = torch.cuda.Event(enable_timing=True)
    e0.record(s_h2d)
    for k in range(e_steps):
        step(k)
    e1 = torch.cuda.Event(enable_timing=True)
    s_d2h.wait_stream(stream)
    e1.record(s_d2h)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), dist, device)
    del ad, bd
    return {"value": job_units * e_steps / (e2e_ms * 1e-3) / scale, "unit": unit,
            "h2d_bytes_per_step": a_h.numel() * a_h.element_size() + b_h.numel() * b_h.element_size(),
            "d2h_bytes_per_step": out_h.numel() * 4, "steps": e_steps,
            "note": "per rank; value = the job's work per step x steps / max-over-ranks time"}


def measure_cpu_path(name, args):
    """A config on the product's device="cpu" path (config 1 is defined there):
    wall-clock time of the synchronous host runner, bit-exact parity against the
    oracle, and the reference's own CPU library timed beside it."""
    import numpy as np
    from oracle import oracle
    from pto_einsum import EinsumBuilder
    eq, s0, s1, dt = CFG[name]
    a, b = fullsize.make_inputs(name)
    bld = EinsumBuilder(eq, [s0, s1], getattr(torch, dt), device="cpu")
    run = bld.build()
    for _ in range(3):
        out = run(a, b)
    reps = max(args.steps, 10)
    t0 = time.perf_counter()
    for _ in range(reps):
        out = run(a, b)
    dt_s = (time.perf_counter() - t0) / reps
    w = work(name)
    metric, unit = metric_of(w)
    scale = 1e12 if w["kind"] == "flops" else 1e9
    res = {"device": "cpu (product host path, include/pto_einsum_cpu.h)", "value": w["units"] / dt_s / scale,
           "unit": unit, "ms_per_step": dt_s * 1e3, "steps": reps, "threads": os.cpu_count(),
           "parity": {"bit_exact": bool(np.array_equal(out.numpy(), oracle.einsum_cpu(eq, a, b))),
                      "oracle": "oracle/einsum_oracle.c (restates the reference include/cpu_einsum.h:53-92)"}}
    r = cpu_reference(name)
    if r:
        res["cpu_baseline"] = {"value": r[0], "unit": unit, "cores": r[1], "kind": "reference", "sample": r[2]}
    bld.cleanup()
    return res


def measure_gather(name, args, rank, world, dist, device):
    """Optional result-on-every-rank path: sharded_einsum(gather=True) (this
    rank's shard, then one NCCL all-gather over NVLink), timed on its own
    against the shard compute alone. Max over ranks."""
    from pto_einsum.distributed import shard_operands, shard_plan, sharded_einsum
    eq = CFG[name][0]
    a, b = fullsize.make_inputs(name, device=device)
    full_size = shard_plan(eq, a.shape, b.shape)[3]
    a, b = shard_operands(eq, a, b, rank, world)
    from pto_einsum import EinsumBuilder
    run = EinsumBuilder(eq, [a.shape, b.shape], a.dtype, device=device).build()
    compute = lambda e, x, y: run(x, y)  # noqa: E731
    reps = 10
    for _ in range(3):
        sharded_einsum(eq, a, b, full_size=full_size, gather=True, compute=compute)
    _barrier(dist, device)
    t_compute = _max_over_ranks(_time(lambda: run(a, b), reps, 2), dist, device)
    _barrier(dist, device)
    t_gather = _max_over_ranks(_time(lambda: sharded_einsum(eq, a, b, full_size=full_size, gather=True,
                                                            compute=compute), reps, 2), dist, device)
    full_out = sharded_einsum(eq, a, b, full_size=full_size, gather=True, compute=compute)
    nbytes = full_out.numel() * 4
    return {"ms_compute_shard": t_compute, "ms_compute_and_allgather": t_gather,
            "ms_allgather": t_gather - t_compute, "output_bytes": nbytes,
            "allgather_busbw_GBps": nbytes * (world - 1) / world / ((t_gather - t_compute) * 1e-3) / 1e9
            if t_gather > t_compute else None,
            "how": "sharded_einsum(gather=True): shard einsum + NCCL all_gather of padded shards + trim; "
                   "CUDA events, 10 calls, max over ranks"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2", choices=sorted(CFG))
    ap.add_argument("--configs", default="all",
                    help="also measure these configs into the line's `configs` map: all, none, or a comma list")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=16,
                    help="pipelined end-to-end steps (fill and drain cost about one step)")
    ap.add_argument("--suite", default=None, choices=["callers", "permute", "gdn", "kda", "base", "thin", "host", "phases"],
                    help="instead of the one-line benchmark: one JSON line per op of that suite")
    ap.add_argument("--sustained-ms", type=float, default=1000.0,
                    help="length of the sustained back-to-back run after the timed region (0: K steps only)")
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
    suites = {"callers": run_callers_suite, "permute": run_permute_suite, "gdn": run_gdn_suite,
              "kda": run_kda_suite,
              "base": run_base_suite, "thin": run_thin_suite, "host": run_host_suite,
              "phases": run_phases_suite}
    if args.suite:
        suites[args.suite](args)
        return

    t_main = time.time()
    dist = None
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        # one kernel cache per rank: ranks build the same libraries and clean up
        # after themselves
        base = os.environ.get("EINSUM_BUILD_DIR") or os.path.join(os.getcwd(), "build")
        os.environ["EINSUM_BUILD_DIR"] = os.path.join(base, f"rank{rank}")
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device)
    clocks = Clocks(device)
    clocks.start()
    time.sleep(0.2)

    name = args.config
    want_cpu = not args.no_cpu_baseline
    head = measure(name, args, rank, world, dist, device, clocks, steps=args.steps, cpu=want_cpu,
                   parity=not args.no_parity)
    extra = {}
    if world > 1:
        weak = measure(name, args, rank, world, dist, device, clocks, steps=args.steps, shard=False,
                       parity=False, e2e=False)
        extra["weak_scaling"] = {"value": weak["value"], "unit": weak["unit"], "ms_per_step": weak["ms_per_step"],
                                 "global_batch": CFG[name][1][0] * world,
                                 "how": "every rank runs the whole config (no sharding), max-over-ranks time"}
        extra["allgather"] = measure_gather(name, args, rank, world, dist, device)
    others = []
    if args.configs != "none":
        others = [n for n in CFG if n != name and n != "cfg1"] if args.configs == "all" else \
            [n for n in args.configs.split(",") if n and n != name]
    cmap = {}
    # At N > 1 the other configs are timed without their end-to-end, parity and
    # sustained extras (those are per-GPU properties measured at N = 1), so the
    # scaling runs hold the GPUs briefly.
    light = world > 1
    for n in others:
        cmap[n] = measure(n, args, rank, world, dist, device, clocks, steps=args.steps, cpu=want_cpu,
                          parity=not args.no_parity and not light, e2e=not light,
                          sustained_ms=0 if light else min(args.sustained_ms, 500.0))
    if world == 1 and args.configs != "none":
        cmap["cfg1"] = measure_cpu_path("cfg1", args)
    clocks.stop()

    if rank == 0:
        lead = CFG[name][1][0]
        line = {
            "metric": head["metric"], "value": head["value"], "unit": head["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": head["dtype"],
            "data": "synthetic (seeded, generated on the device)",
            "config": dict(head["config"], global_batch=lead,
                           parallelism=f"leading axis sharded over {world} GPU(s) "
                                       "(pto_einsum.distributed.shard_operands), no collective on the data path"),
            "roofline": head["roofline"], "cpu_baseline": head.get("cpu_baseline"), "e2e": head["e2e"],
            "parity": head.get("parity"), "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
            "sustained": head["sustained"], "library_reference": head.get("library_reference"),
        }
        line.update(extra)
        line["bench_wall_s"] = round(time.time() - t_main, 1)
        if cmap:
            line["configs"] = {n: {k: v for k, v in r.items() if k not in ("metric",)} for n, r in cmap.items()}
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
