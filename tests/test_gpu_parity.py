"""CUDA path vs the CPU oracle on the reference's parity corpus (GPU)."""
import ctypes
import math
import zlib

import numpy as np
import pytest
import torch

from corpus import ATTENTION_CASES, BROADCAST_CASES, CHAIN_CASES, EINSUM_CASES, BATCHED_PARTIAL, case_id
from gpu_util import TOL, check_close, seeded
from oracle import oracle
from pto_einsum import EinsumBuilder, einsum, planner
from pto_einsum import _core

pytestmark = pytest.mark.gpu

CONTRACTIONS = EINSUM_CASES + ATTENTION_CASES + CHAIN_CASES + BATCHED_PARTIAL
DTYPES = [torch.float32, torch.float16]


def _is_exact(eq, s0, s1):
    r, _ = planner.choose_operand_order("cuda", eq, s0, s1)
    return r["elementwise"] or r["broadcast"]


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
@pytest.mark.parametrize("eq,s0,s1", CONTRACTIONS + BROADCAST_CASES,
                         ids=[case_id(*c) for c in CONTRACTIONS + BROADCAST_CASES])
def test_einsum_matches_oracle(eq, s0, s1, dtype):
    seed = zlib.crc32(repr((eq, s0, s1)).encode()) % 10000
    a, b = seeded(s0, dtype, seed), seeded(s1, dtype, seed + 1)
    out = einsum(eq, a.cuda(), b.cuda())
    assert out.dtype == torch.float32 and out.device.type == "cuda"
    ref = oracle.einsum_cpu(eq, a, b)
    check_close(out, ref, dtype, exact=_is_exact(eq, s0, s1))
    # torch.einsum tolerance of the reference suite (tests/test_einsum.py:143-154)
    tol = 1e-4 if dtype == torch.float32 else 1e-2
    exp = torch.einsum(eq, a.float(), b.float())
    torch.testing.assert_close(out.cpu(), exp, rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
@pytest.mark.parametrize("eq,s0,s1", [
    ("bij, bjk -> bik", (64, 128, 128), (64, 128, 128)),
    ("bihd, bjhd -> bihj", (2, 128, 16, 128), (2, 128, 16, 128)),
    ("bihj, bjhd -> bihd", (2, 128, 16, 128), (2, 128, 16, 128)),
    ("bvhd, bvhe -> bhde", (2, 128, 16, 128), (2, 128, 16, 128)),
    ("ji, jk -> ik", (512, 500), (512, 64)),
])
def test_bit_exact_reruns(eq, s0, s1, dtype):
    """Race detector (tests/test_einsum.py:245-364): 8 reruns on the same input
    must be bit-identical."""
    b = EinsumBuilder(eq, [s0, s1], dtype)
    run = b.build()
    x, y = seeded(s0, dtype, 11).cuda(), seeded(s1, dtype, 12).cuda()
    first = run(x, y).clone()
    check_close(first, oracle.einsum_cpu(eq, x.cpu(), y.cpu()), dtype)
    for _ in range(8):
        assert torch.equal(run(x, y), first)
    b.cleanup()


SPLITK_CASES = [  # thin outputs, long contractions: split-K partials + reduce
    ("ts, sp -> tp", (512, 8192), (8192, 128)),
    ("ij, jk -> ik", (16, 4096), (4096, 16)),
    ("bij, bjk -> bik", (2, 128, 8192), (2, 8192, 96)),
    ("bki, bkj -> ibj", (2, 4096, 64), (2, 4096, 48)),
]


STREAMK_CASES = SPLITK_CASES + [  # forced stream-K on short contractions: ragged tiles,
    ("ij, jk -> ik", (300, 1000), (1000, 200)),              # batches, permuted outputs
    ("bij, bjk -> bik", (3, 130, 520), (3, 520, 72)),
    ("bhsd, bhtd -> bsht", (1, 2, 128, 256), (1, 2, 128, 256)),
    ("ki, kj -> ji", (2048, 96), (2048, 200)),
]


@pytest.mark.parametrize("mode", ["auto", "splitk", "streamk"])
@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
@pytest.mark.parametrize("eq,s0,s1", STREAMK_CASES, ids=[case_id(*c) for c in STREAMK_CASES])
def test_split_k(eq, s0, s1, dtype, mode, monkeypatch):
    """Thin outputs with long contractions: split-K slabs (PE_GEMM_STREAMK=0),
    stream-K segments (=2, forced wherever it applies) and the default choice.
    Each must match the oracle and be bit-identical over reruns."""
    if mode == "splitk":
        monkeypatch.setenv("PE_GEMM_STREAMK", "0")
    elif mode == "streamk":
        monkeypatch.setenv("PE_GEMM_STREAMK", "2")
    b = EinsumBuilder(eq, [s0, s1], dtype)
    run = b.build()
    x, y = seeded(s0, dtype, 21, "randn"), seeded(s1, dtype, 22, "randn")
    first = run(x.cuda(), y.cuda()).clone()
    check_close(first, oracle.einsum_cpu(eq, x, y), dtype)
    for _ in range(3):
        assert torch.equal(run(x.cuda(), y.cuda()), first)
    b.cleanup()


THIN_CASES = [  # thin outputs over a contiguous contraction: warp-per-dot streaming kernel
    ("i, i ->", (256,), (256,)), ("i, i ->", (1001,), (1001,)), ("i, i ->", (131072,), (131072,)),
    ("ij, j -> i", (256, 4096), (4096,)), ("ij, j -> i", (3, 5000), (5000,)), ("ij, j -> i", (1000, 300), (300,)),
    ("bij, bj -> bi", (4, 64, 4096), (4, 4096)), ("ij, kj -> ik", (96, 2048), (3, 2048)),
    ("bhd, bhd -> bh", (8, 32, 1024), (8, 32, 1024)), ("j, ij -> i", (4104,), (7, 4104)),
    ("ijk, ijk ->", (4, 16, 300), (4, 16, 300)),
]


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
@pytest.mark.parametrize("eq,s0,s1", THIN_CASES, ids=[case_id(*c) for c in THIN_CASES])
def test_thin_contraction(eq, s0, s1, dtype):
    b = EinsumBuilder(eq, [s0, s1], dtype)
    run = b.build()
    x, y = seeded(s0, dtype, 51, "randn"), seeded(s1, dtype, 52, "randn")
    first = run(x.cuda(), y.cuda()).clone()
    r = planner.choose_operand_order("cuda", eq, s0, s1)[0]
    if r["C"] <= 8192:
        # the oracle sums sequentially in fp32: itself accurate only for short sums
        check_close(first, oracle.einsum_cpu(eq, x, y), dtype)
    # per element: |out - exact| <= 1e-6 * sum |a_i b_i| (the dot product's condition)
    exact = torch.einsum(eq, x.double(), y.double())
    scale = torch.einsum(eq, x.double().abs(), y.double().abs())
    assert ((first.cpu().double() - exact).abs() <= 1e-6 * scale + 1e-30).all()
    for _ in range(3):
        assert torch.equal(run(x.cuda(), y.cuda()), first)
    b.cleanup()


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
def test_thin_long_dot_and_misaligned(dtype):
    """64M-element dot product (many chunk partials) and a misaligned operand
    base (scalar loads) against float64."""
    n = 1 << 26
    g = torch.Generator(device="cuda").manual_seed(61)
    a = torch.randn(n + 1, device="cuda", generator=g).to(dtype)
    b = torch.randn(n, device="cuda", generator=g).to(dtype)
    for x in (a[:n], a[1:]):
        out = einsum("i, i ->", x, b)
        ref = (x.double() * b.double()).sum()
        assert abs(out.item() - ref.item()) <= 1e-6 * (x.double().abs() * b.double().abs()).sum().item()


def test_streamk_full_size_cfg4c():
    """Config 4c ('ts,sp->tp', fp32, 8192 x 8192 x 128: 64 tiles on 148 SMs), which
    the cost model runs as stream-K: vs float64 on the GPU."""
    eq, s0, s1 = "ts, sp -> tp", (8192, 8192), (8192, 128)
    g = torch.Generator(device="cuda").manual_seed(41)
    a = torch.randn(s0, device="cuda", generator=g)
    b = torch.randn(s1, device="cuda", generator=g)
    out = einsum(eq, a, b)
    ref = a.double() @ b.double()
    err = ((out.double() - ref).norm() / ref.norm()).item()
    assert err <= 1e-5, err
    assert torch.equal(einsum(eq, a, b), out)


def test_fp32_long_positive_contraction():
    """All-positive data, K = 8192: the worst case for the tensor core's fp32
    accumulation (errors do not cancel); 4 interleaved accumulators keep it
    within the fp32 tolerance."""
    eq, s0, s1 = "ij, jk -> ik", (256, 8192), (8192, 256)
    a, b = seeded(s0, torch.float32, 31), seeded(s1, torch.float32, 32)
    check_close(einsum(eq, a.cuda(), b.cuda()), oracle.einsum_cpu(eq, a, b), torch.float32)


def test_tf32_truncation_mode_is_exact(monkeypatch):
    """The default 3xTF32 split feeds raw fp32 data as the tf32 "big" part
    (the tensor core ignores the low 13 mantissa bits); it must give the same
    bits as writing back the explicitly masked value."""
    for eq, s0, s1 in [("ij, jk -> ik", (256, 1024), (1024, 256)), ("ts, sp -> tp", (512, 4096), (4096, 128)),
                       ("ji, jk -> ik", (200, 96), (200, 136))]:
        a, b = seeded(s0, torch.float32, 41, "randn").cuda(), seeded(s1, torch.float32, 42, "randn").cuda()
        monkeypatch.setenv("PE_TF32_HW_TRUNC", "0")
        masked = einsum(eq, a, b)
        monkeypatch.setenv("PE_TF32_HW_TRUNC", "1")
        raw = einsum(eq, a, b)
        assert torch.equal(masked, raw)


def test_builder_reuse_workspace():
    """Persistent workspace reused across calls with fresh data
    (tests/test_einsum.py:208-241), including a gathered (K != C) operand."""
    for eq, s0, s1 in [("ij, jk -> ik", (32, 64), (64, 32)), ("bij, bjk -> bik", (8, 16, 20), (8, 20, 64)),
                       ("bhsc, bcht -> bsht", (2, 8, 16, 20), (2, 20, 8, 24))]:
        run = EinsumBuilder(eq, [s0, s1], torch.float32).build()
        for k in range(10):
            a, b = seeded(s0, torch.float32, 100 + k), seeded(s1, torch.float32, 200 + k)
            check_close(run(a.cuda(), b.cuda()), oracle.einsum_cpu(eq, a, b), torch.float32)


def test_guard_bands_untouched():
    """Out-of-bounds canary: the output sits between NaN guard bands that must
    survive every route (elementwise, broadcast, direct GEMM, gathered GEMM,
    strided epilogue)."""
    cases = [("ij,jk->ik", (250, 128), (128, 250), torch.float32),
             ("bshd,bthd->bsht", (2, 64, 4, 32), (2, 96, 4, 32), torch.float16),
             ("ij,jk->ki", (32, 64), (64, 48), torch.float32),
             ("ts,ts->ts", (63, 47), (63, 47), torch.float16),
             ("bshd,sd->bshd", (2, 8, 4, 16), (8, 16), torch.float16),
             ("bhsc,bhtc->bhst", (2, 4, 16, 130), (2, 4, 256, 130), torch.float32)]
    guard = 4096
    for eq, s0, s1, dt in cases:
        b = EinsumBuilder(eq, [s0, s1], dt)
        b.build()
        n = int(np.prod(b.recipe["out_shape"]))
        buf = torch.full((guard + n + guard,), float("nan"), device="cuda")
        x, y = seeded(s0, dt, 5).cuda(), seeded(s1, dt, 6).cuda()
        if b._swap_operands:
            x, y = y, x
        stream = torch.cuda.current_stream().cuda_stream
        ws = b.workspace(x.device, stream)
        P = ctypes.POINTER
        b.lib.run_einsum_exec(ctypes.cast(x.data_ptr(), P(b.c_type)), ctypes.cast(y.data_ptr(), P(b.c_type)),
                              ctypes.cast(buf.data_ptr() + 4 * guard, P(ctypes.c_float)), ctypes.c_void_p(ws),
                              ctypes.c_void_p(stream))
        assert b.lib.run_einsum_last_error() == 0
        torch.cuda.synchronize()
        assert torch.isnan(buf[:guard]).all() and torch.isnan(buf[guard + n:]).all()
        assert not torch.isnan(buf[guard:guard + n]).any()
        b.cleanup()


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
def test_standalone_entry_points(dtype):
    """run_transpose_inp0/inp1/out and run_batched_matmul
    (tests/test_matmul.py:24-151): each stage against the oracle."""
    eq, s0, s1 = "bhsc, bcht -> bsht", (2, 8, 16, 20), (2, 20, 8, 24)
    b = EinsumBuilder(eq, [s0, s1], dtype)
    b.build()
    r = b.recipe
    x, y = seeded(s0, dtype, 1), seeded(s1, dtype, 2)
    if b._swap_operands:
        x, y = y, x
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = ctypes.POINTER
    ptr = lambda t, ct: ctypes.cast(t.data_ptr(), P(ct))  # noqa: E731
    p0, p1 = r["in_transpose_idxs"]
    t0 = torch.empty([x.shape[i] for i in p0], dtype=dtype, device="cuda")
    t1 = torch.empty([y.shape[i] for i in p1], dtype=dtype, device="cuda")
    xc, yc = x.cuda(), y.cuda()
    b.lib.run_transpose_inp0(ptr(xc, b.c_type), ptr(t0, b.c_type), stream)
    b.lib.run_transpose_inp1(ptr(yc, b.c_type), ptr(t1, b.c_type), stream)
    torch.cuda.synchronize()
    assert torch.equal(t0.cpu(), x.permute(p0).contiguous())
    assert torch.equal(t1.cpu(), y.permute(p1).contiguous())
    I, L0, L1, C = r["I"], r["L0"], r["L1"], r["C"]
    res = torch.empty((I, L0, L1), dtype=torch.float32, device="cuda")
    b.lib.run_batched_matmul(ptr(t0, b.c_type), ptr(t1, b.c_type), ptr(res, ctypes.c_float), stream)
    torch.cuda.synchronize()
    assert b.lib.run_einsum_last_error() == 0
    ref_mm = oracle.batched_matmul_cpu(t0.cpu().reshape(I, L0, C), t1.cpu().reshape(I, C, L1))
    check_close(res, ref_mm, dtype)
    out = torch.empty(r["out_shape"], dtype=torch.float32, device="cuda")
    b.lib.run_transpose_out(ptr(res, ctypes.c_float), ptr(out, ctypes.c_float), stream)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), res.cpu().reshape(r["out_interpret_shape"]).permute(r["out_transpose_idxs"]))
    b.cleanup()


TRANSPOSE_CASES = [  # tests/test_transpose.py:108-162 (shape, perm)
    ((128,), (0,)), ((32, 64), (0, 1)), ((8, 16, 32), (0, 1, 2)), ((4, 8, 16, 32), (0, 1, 2, 3)),
    ((123,), (0,)), ((17, 35), (0, 1)), ((3, 7, 13), (0, 1, 2)), ((32, 64), (1, 0)), ((16, 16), (1, 0)),
    ((10, 20), (1, 0)), ((8, 12), (1, 0)), ((256, 256), (1, 0)), ((512, 64), (1, 0)), ((80, 256), (1, 0)),
    ((144, 208), (1, 0)), ((201, 199), (1, 0)), ((333, 257), (1, 0)), ((257, 257), (1, 0)),
    ((2, 3, 4, 5), (3, 1, 0, 2)), ((8, 33, 2, 65), (0, 3, 1, 2)),
    # kernel-path coverage: vector run copy with outer decode, odd runs,
    # 128-wide 2-byte tiles with ragged edges, narrow destination axis
    ((4, 40, 8, 16), (0, 2, 1, 3)), ((4, 6, 5, 7), (0, 2, 1, 3)), ((136, 392), (1, 0)),
    ((3, 200, 136), (0, 2, 1)), ((2, 64, 32, 128), (3, 1, 0, 2)), ((2, 24, 4, 136), (0, 2, 3, 1)),
    ((40, 24, 16), (1, 2, 0)), ((6, 48, 8, 24), (1, 3, 0, 2)),
]


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
@pytest.mark.parametrize("shape,perm", TRANSPOSE_CASES)
def test_permute_kernel(shape, perm, dtype):
    lib = _core.core_lib()

    class Plan(ctypes.Structure):
        _fields_ = [("dtype", ctypes.c_int32), ("dims", ctypes.c_int32),
                    ("from_shape", ctypes.c_int64 * 8), ("perm", ctypes.c_int32 * 8)]
    p = Plan()
    p.dtype = 0 if dtype == torch.float32 else 1
    p.dims = len(shape)
    for i, (s, q) in enumerate(zip(shape, perm)):
        p.from_shape[i] = s
        p.perm[i] = q
    x = seeded(shape, dtype, 9).cuda()
    out = torch.empty([shape[i] for i in perm], dtype=dtype, device="cuda")
    rc = lib.pe_permute(ctypes.byref(p), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    assert torch.equal(out, x.permute(perm).contiguous())


def _fuzz_permute_cases(n=24, seed=5):
    import random
    rng = random.Random(seed)
    cases = []
    for _ in range(n):
        nd = rng.randint(2, 5)
        shape = tuple(rng.choice([1, 2, 3, 8, 16, 24, 40, 64, 72, 136]) for _ in range(nd))
        while math.prod(shape) > (1 << 21):
            shape = tuple(max(1, v // 2) for v in shape)
        perm = list(range(nd))
        rng.shuffle(perm)
        cases.append((shape, tuple(perm)))
    return cases


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
@pytest.mark.parametrize("shape,perm", _fuzz_permute_cases())
def test_permute_kernel_fuzz(shape, perm, dtype):
    """Seeded random shapes and permutations through every copy path (run copy,
    tiled transposes with and without widened axes, element copy): exact."""
    test_permute_kernel(shape, perm, dtype)


def test_zero_size_and_degenerate():
    # empty batch -> empty output; zero contraction -> zeros
    out = einsum("bij,bjk->bik", torch.rand(0, 4, 8, device="cuda"), torch.rand(0, 8, 5, device="cuda"))
    assert out.shape == (0, 4, 5)
    out = einsum("ij,jk->ik", torch.rand(4, 0, device="cuda"), torch.rand(0, 5, device="cuda"))
    assert torch.equal(out, torch.zeros(4, 5, device="cuda"))
    out = einsum("i,i->", torch.rand(256, device="cuda"), torch.rand(256, device="cuda"))
    assert out.shape == ()


def test_no_device_errors_and_native_launches():
    before = _core.launch_count()
    einsum("ij,jk->ik", torch.rand(64, 64, device="cuda"), torch.rand(64, 64, device="cuda"))
    assert _core.launch_count() > before
    assert _core.device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_validation_errors_cuda():
    a, b = torch.rand(32, 64, device="cuda"), torch.rand(64, 32, device="cuda")
    with pytest.raises(ValueError, match="Only exactly two operands are supported."):
        einsum("ij,jk->ik", a)
    with pytest.raises(ValueError, match="Operands must have the same datatype."):
        einsum("ij,jk->ik", a, b.to(torch.int32))
    run = EinsumBuilder("ij,jk->ik", [(32, 64), (64, 32)], torch.float32).build()
    with pytest.raises(ValueError, match="do not match built shapes"):
        run(torch.rand(32, 32, device="cuda"), b)
    with pytest.raises(TypeError, match="do not match built datatype"):
        run(a, b.half())
    with pytest.raises(ValueError, match="same CUDA device"):
        run(a.cpu(), b.cpu())


PAIR_CASES = [  # fp16 shapes with >= 148 wide (256-column) tiles: the CTA-pair kernel
    ("bij, bjk -> bik", (40, 512, 512), (40, 512, 512)),     # B MN-major
    ("bij, bjk -> bik", (40, 300, 136), (40, 136, 520)),     # partial M and N tiles, K not a tile multiple
    ("bshd, bthd -> bsht", (4, 512, 8, 512), (4, 512, 8, 512)),  # B K-major, permuted output
    ("bik, bjk -> bij", (24, 384, 256), (24, 768, 256)),     # K-major both
]


@pytest.mark.parametrize("eq,s0,s1", PAIR_CASES, ids=[case_id(*c) for c in PAIR_CASES])
def test_cta_pair_kernel(eq, s0, s1, monkeypatch):
    """tcgen05 cta_group::2 tiles (two CTAs per 256x256 tile) against the oracle
    and against the single-CTA kernel."""
    a, b = seeded(s0, torch.float16, 51, "randn"), seeded(s1, torch.float16, 52, "randn")
    ref = oracle.einsum_cpu(eq, a, b)
    monkeypatch.setenv("PE_GEMM_PAIRS", "1")
    pair = einsum(eq, a.cuda(), b.cuda())
    check_close(pair, ref, torch.float16)
    for _ in range(3):
        assert torch.equal(einsum(eq, a.cuda(), b.cuda()), pair)
    monkeypatch.setenv("PE_GEMM_PAIRS", "0")
    single = einsum(eq, a.cuda(), b.cuda())
    check_close(single, ref, torch.float16)
    torch.testing.assert_close(pair, single, rtol=1e-5, atol=1e-5)
    assert _core.device_error(torch.cuda.current_stream().cuda_stream) == 0


from llm_patterns import PATTERNS, SMALL, shapes as llm_shapes  # noqa: E402


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16"])
@pytest.mark.parametrize("name,eq", PATTERNS, ids=[p[0] for p in PATTERNS])
def test_llm_patterns(name, eq, dtype):
    """The reference's LLM contraction patterns (bench_llm_contractions.py) at
    small sizes, against the CPU oracle."""
    s0, s1 = llm_shapes(eq, SMALL)
    a, b = seeded(s0, dtype, 61, "randn"), seeded(s1, dtype, 62, "randn")
    out = einsum(eq, a.cuda(), b.cuda())
    check_close(out, oracle.einsum_cpu(eq, a, b), dtype, exact=_is_exact(eq, s0, s1))


@pytest.mark.parametrize("eq,s0,s1", [("tn, sn -> ts", (2048, 128), (4096, 128)),
                                      ("ij, jk -> ik", (1000, 96), (96, 5000))])
def test_fp32_wide_tiles(eq, s0, s1, monkeypatch):
    """fp32 with both tf32 small halves precomputed on 256-column tiles, against
    the oracle and the 128-column kernel."""
    a, b = seeded(s0, torch.float32, 71, "randn"), seeded(s1, torch.float32, 72, "randn")
    ref = oracle.einsum_cpu(eq, a, b)
    monkeypatch.setenv("PE_GEMM_WIDE_FP32", "1")
    wide = einsum(eq, a.cuda(), b.cuda())
    check_close(wide, ref, torch.float32)
    monkeypatch.setenv("PE_GEMM_WIDE_FP32", "0")
    narrow = einsum(eq, a.cuda(), b.cuda())
    check_close(narrow, ref, torch.float32)
    assert _core.device_error(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("eq,s0,s1", [("tn, sn -> ts", (4096, 128), (4096, 128)),
                                      ("tn, sn -> ts", (4000, 96), (3000, 96)),
                                      ("bik, bjk -> bij", (8, 1024, 64), (8, 1000, 64))])
def test_fp32_cta_pairs_match_single_cta_and_oracle(eq, s0, s1, monkeypatch):
    """3xTF32 on CTA pairs (256x256 tiles, both tf32 small halves precomputed)
    against the single-CTA wide kernel (PE_GEMM_FP32_PAIRS=0) and the oracle,
    with ragged row and column tiles."""
    a, b = seeded(s0, torch.float32, 3, "randn"), seeded(s1, torch.float32, 4, "randn")
    ref = oracle.einsum_cpu(eq, a, b)
    outs = []
    for flag in ("1", "0"):
        monkeypatch.setenv("PE_GEMM_FP32_PAIRS", flag)
        bld = EinsumBuilder(eq, [s0, s1], torch.float32)
        out = bld.build()(a.cuda(), b.cuda())
        check_close(out, ref, torch.float32)
        outs.append(out)
        bld.cleanup()
    assert _core.device_error(torch.cuda.current_stream().cuda_stream) == 0
