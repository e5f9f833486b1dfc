"""Host-side fault injection (no GPU fault is ever provoked): a missing
compiler, a damaged cache entry, a host allocation failure under a memory cap,
a shape/dtype mismatch, a device workspace allocation that cannot succeed, and
a rank that dies before the optional all-gather. Each must fail loudly (an
exception naming the problem) or recover, never hang or return garbage. The
reference's contract is loud errors only (src/pto_einsum/builder.py:155-183,
:613, :735-736)."""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from oracle import oracle
from pto_einsum import EinsumBuilder

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_missing_compiler_is_a_runtime_error(monkeypatch):
    monkeypatch.setenv("CXX", "/nonexistent/bin/g++")
    b = EinsumBuilder("ij,jk->ik", [(8, 16), (16, 8)], torch.float32, device="cpu")
    b.parse_equation()
    b.generate_code()
    b.code_hash = "f" * 32                      # force a cache miss
    b.target_dir = os.path.join(b.build_base, b.code_hash)
    with pytest.raises(RuntimeError, match="cannot run the compiler"):
        b.compile()
    b.cleanup()


@pytest.mark.parametrize("damage", ["garbage", "truncated", "empty"])
def test_damaged_cache_entry_is_rebuilt(damage):
    eq, s0, s1 = "ij,jk->ik", (24, 40), (40, 16)
    first = EinsumBuilder(eq, [s0, s1], torch.float32, device="cpu")
    first.parse_equation()
    first.generate_code()
    first.compile()                               # cached, never loaded by this process
    so = first.so_filename
    data = open(so, "rb").read()
    with open(so, "wb") as f:
        f.write({"garbage": b"\x7fELF not really a library" * 100,
                 "truncated": data[: len(data) // 3], "empty": b""}[damage])
    b = EinsumBuilder(eq, [s0, s1], torch.float32, device="cpu")
    run = b.build()                               # load fails once, the entry is rebuilt
    g = torch.Generator().manual_seed(1)
    x, y = torch.rand(s0, generator=g), torch.rand(s1, generator=g)
    np.testing.assert_array_equal(run(x, y).numpy(), oracle.einsum_cpu(eq, x, y))
    b.cleanup()


def test_host_allocation_failure_under_memory_cap(tmp_path):
    """device='cpu' under an address-space cap just above what is in use: the
    host library's buffers cannot be allocated and the runner raises
    MemoryError (run in a child process so the cap does not leak)."""
    script = textwrap.dedent(f"""
        import os, resource, sys
        sys.path[:0] = [{os.path.join(REPO, 'pto-einsum_b200')!r}, {REPO!r}]
        os.environ["EINSUM_BUILD_DIR"] = {str(tmp_path)!r}
        import torch
        from pto_einsum import EinsumBuilder
        n = 2048
        run = EinsumBuilder("ij,kj->ik", [(n, n), (n, n)], torch.float32, device="cpu").build()
        a, b = torch.ones(n, n), torch.ones(n, n)
        vm = int([l for l in open("/proc/self/status") if l.startswith("VmSize")][0].split()[1]) * 1024
        # room for the 16 MB output, not for the 48 MB of internal buffers
        resource.setrlimit(resource.RLIMIT_AS, (vm + (24 << 20), resource.RLIM_INFINITY))
        try:
            run(a, b)
        except MemoryError as e:
            print("MEMORYERROR", e)
        except RuntimeError as e:
            print("RUNTIMEERROR", e)
        else:
            print("NOERROR")
    """)
    r = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "MEMORYERROR" in r.stdout or "RUNTIMEERROR" in r.stdout, r.stdout + r.stderr[-2000:]


def test_shape_and_dtype_mismatch_are_loud():
    run = EinsumBuilder("bij,bjk->bik", [(2, 8, 4), (2, 4, 8)], torch.float32, device="cpu").build()
    with pytest.raises(ValueError, match="do not match built shapes"):
        run(torch.zeros(2, 8, 5), torch.zeros(2, 5, 8))
    with pytest.raises(TypeError, match="do not match built datatype"):
        run(torch.zeros(2, 8, 4, dtype=torch.float64), torch.zeros(2, 4, 8, dtype=torch.float64))
    with pytest.raises(ValueError, match="Expected exactly two operands"):
        run(torch.zeros(2, 8, 4))


@pytest.mark.gpu
def test_device_workspace_allocation_failure_is_loud():
    """A plan whose gathered operand needs more scratch than the GPU has (fp16
    rows of 20 elements cannot be read by a tensor map; 4 x 2^30 rows x 48 bytes
    = 206 GB): run_einsum_setup's cudaMalloc fails, the builder raises, and the
    failed allocation does not poison later launches on this thread."""
    from pto_einsum import einsum
    b = EinsumBuilder("bij,bjk->bik", [(4, 1 << 30, 20), (4, 20, 64)], torch.float16)
    b.build()
    dev = torch.device("cuda", torch.cuda.current_device())
    with pytest.raises(RuntimeError, match="run_einsum_setup failed"):
        b.workspace(dev, torch.cuda.current_stream().cuda_stream)
    b.cleanup()
    x = torch.rand(4, 64, 32, device="cuda", dtype=torch.float16)
    y = torch.rand(4, 32, 48, device="cuda", dtype=torch.float16)
    out = einsum("bij,bjk->bik", x, y)
    torch.testing.assert_close(out, torch.bmm(x.float(), y.float()), rtol=2e-3, atol=2e-3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gather_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    from pto_einsum.distributed import shard_operands, shard_plan, sharded_einsum
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    eq, s0, s1 = "bij,bjk->bik", (4, 8, 16), (4, 16, 8)
    a, b = torch.ones(s0), torch.ones(s1)
    al, bl = shard_operands(eq, a, b, rank, world)
    cpu = lambda e, x, y: torch.from_numpy(oracle.einsum_cpu(e, x, y))  # noqa: E731
    if rank == 1:
        q.put((rank, "died"))
        q.close()
        q.join_thread()      # the message is flushed before the process vanishes
        os._exit(3)          # the rank leaves between steps, before the collective
    try:
        sharded_einsum(eq, al, bl, full_size=shard_plan(eq, s0, s1)[3], gather=True, compute=cpu)
        q.put((rank, "no error"))
    except Exception as e:   # gloo reports the lost peer or the timeout
        q.put((rank, f"raised {type(e).__name__}"))


def test_rank_lost_before_gather_raises_not_hangs():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "died"
    assert res[0].startswith("raised"), res
