"""Batch sharding on two GPUs: one NCCL rank per GPU runs its shard through
the CUDA path, then sharded_einsum(gather=True) assembles the full result with
one all-gather. The gathered result must equal the one-GPU result of the same
inputs (bit for bit where the per-tile schedule cannot change with the shard:
no split-K or stream-K), and match the CPU oracle. Skipped with fewer than two
GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = [
    # (equation, shape0, shape1, dtype, bit-identical to one GPU)
    ("bij,bjk->bik", (8, 512, 512), (8, 512, 512), torch.float16, True),
    ("bshd,bthd->bsht", (4, 200, 4, 80), (4, 200, 4, 80), torch.float16, True),
    ("tn,sn->ts", (2048, 128), (2048, 128), torch.float32, True),
    ("ts,sp->tp", (2048, 2048), (2048, 128), torch.float32, False),
    ("hqk,h->hqk", (6, 256, 256), (6,), torch.float16, True),
    ("bsd,d->bsd", (3, 128, 512), (512,), torch.float16, True),
]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    from oracle import oracle
    from pto_einsum import einsum
    from pto_einsum.distributed import shard_operands, shard_plan, sharded_einsum
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    results = []
    for k, (eq, s0, s1, dt, same) in enumerate(CASES):
        g = torch.Generator().manual_seed(100 + k)
        a = torch.randn(s0, generator=g).to(dt)
        b = torch.randn(s1, generator=g).to(dt)
        al, bl = shard_operands(eq, a, b, rank, world)
        full = shard_plan(eq, s0, s1)[3]
        out = sharded_einsum(eq, al.to(dev), bl.to(dev), full_size=full, gather=True)
        one = einsum(eq, a.to(dev), b.to(dev))
        got = out.cpu().numpy()
        ref = oracle.einsum_cpu(eq, a, b)
        err = oracle.rel_frobenius(got, ref)
        tol = 1e-5 if dt == torch.float32 else 2e-3
        identical = bool(torch.equal(out, one))
        results.append((eq, err <= tol, identical or not same, err, identical))
    q.put((rank, results))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_gather_matches_one_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, rows in res:
        for eq, ok_tol, ok_same, err, identical in rows:
            assert ok_tol, (rank, eq, err)
            assert ok_same, (rank, eq, "gathered result differs from the one-GPU result")
