"""Batch sharding host logic on CPU with world_size-2 gloo ranks (the CUDA
compute is replaced by the CPU oracle; the shard / gather plumbing is the
product code)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pto_einsum.distributed import shard_bounds, shard_operands, shard_plan, sharded_einsum


def test_shard_bounds_cover_exactly():
    for n in (0, 1, 7, 8, 64, 65):
        for w in (1, 2, 4, 8):
            spans = [shard_bounds(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[r][1] == spans[r + 1][0] for r in range(w - 1))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1


def test_shard_plan_configs():
    assert shard_plan("bij,bjk->bik", (64, 8, 8), (64, 8, 8))[1:] == (0, 0, 64)
    assert shard_plan("tn,sn->ts", (8192, 128), (8192, 128))[1:] == (0, None, 8192)
    assert shard_plan("hqk,h->hqk", (32, 4, 4), (32,))[1:] == (0, 0, 32)
    assert shard_plan("bshd,sd->bshd", (16, 4, 2, 8), (4, 8))[1:] == (0, None, 16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, eq, s0, s1, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import oracle
    g = torch.Generator().manual_seed(0)
    a = torch.randn(s0, generator=g)
    b = torch.randn(s1, generator=g)
    al, bl = shard_operands(eq, a, b, rank, world)
    cpu = lambda e, x, y: torch.from_numpy(oracle.einsum_cpu(e, x, y))  # noqa: E731
    full = shard_plan(eq, s0, s1)[3]
    local = sharded_einsum(eq, al, bl, full_size=full, gather=False, compute=cpu)
    lo, hi = shard_bounds(full, world, rank)
    ref = oracle.einsum_cpu(eq, a, b)
    ok_local = np.array_equal(local.numpy(), ref[lo:hi])
    out = sharded_einsum(eq, al, bl, full_size=full, gather=True, compute=cpu)
    ok_full = np.array_equal(out.numpy(), ref)
    q.put((rank, ok_local, ok_full))
    dist.destroy_process_group()


@pytest.mark.parametrize("eq,s0,s1", [("bij,bjk->bik", (5, 8, 16), (5, 16, 8)),
                                      ("bij,bjk->bik", (4, 8, 16), (4, 16, 8)),
                                      ("tn,sn->ts", (9, 16), (12, 16)),
                                      ("hqk,h->hqk", (3, 4, 4), (3,))])
def test_gloo_two_ranks(eq, s0, s1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, eq, s0, s1, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok_l and ok_f for _, ok_l, ok_f in res), res
