"""KDA caller (pto_einsum.kda): the chunked stages against the step recurrence (CPU),
the B200 contraction backend against torch.einsum and float64 (GPU), CUDA-graph
replay. Mirrors the reference's KDA checks (benchmarks/complex/kda/bench_kda_4way.py
comparing the einsum backends on one glue; tolerance utils.py:8-14, ftol 1e-3)."""
import pytest
import torch

from pto_einsum import _core
from pto_einsum.kda import KDAChunked, KDAGraph, kda_recurrent_reference, random_kda_inputs


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("B,T,H,Hk,D,C,gate", [(1, 96, 2, 2, 8, 32, 0.05), (2, 128, 4, 2, 16, 32, 0.5),
                                               (1, 64, 3, 1, 8, 16, 1.0)])
def test_chunked_matches_recurrence_fp64(B, T, H, Hk, D, C, gate):
    q, k, v, g, beta = random_kda_inputs(T, H, Hk, D, B=B, seed=T + H, dtype=torch.float64, gate=gate)
    o = KDAChunked("torch", chunk=C, dtype=torch.float64)(q, k, v, g, beta, scale=D ** -0.5)
    r = kda_recurrent_reference(q, k, v, g, beta, scale=D ** -0.5)
    assert rel(o, r) < 1e-12


def test_chunked_fp32_final_state_and_folding():
    q, k, v, g, beta = random_kda_inputs(128, 4, 2, 16, B=2, seed=9)
    m = KDAChunked("torch", chunk=32)
    o, S = m(q, k, v, g, beta, return_state=True)
    assert rel(o, kda_recurrent_reference(q, k, v, g, beta)) < 1e-5
    assert S.shape == (2, 4, 16, 16)
    flat = [x.reshape(1, 256, *x.shape[2:]) for x in (q, k, v, g, beta)]
    o1 = m(*flat, cu_seqlens=[0, 128, 256])
    assert rel(o1.reshape(o.shape), o) == 0.0


def test_gate_shape_is_checked():
    q, k, v, g, beta = random_kda_inputs(64, 2, 2, 8, seed=1)
    with pytest.raises(ValueError, match="one log-decay per key dimension"):
        KDAChunked("torch", chunk=32)(q, k, v, g[..., 0], beta)


# ---------------------------------------------------------------------------- GPU
GPU_CASES = [  # (N_seq, L_seg, H, Hk): chunk 128, head dim 128, like the reference's 4-way bench
    (1, 256, 4, 2), (2, 256, 4, 4), (1, 512, 8, 4),
]


@pytest.mark.gpu
@pytest.mark.parametrize("N,L,H,Hk", GPU_CASES)
def test_pto_backend_matches_torch_and_fp64(N, L, H, Hk):
    dev = torch.device("cuda", 0)
    q, k, v, g, beta = random_kda_inputs(N * L, H, Hk, 128, seed=N * L + H, device=dev)
    cu = list(range(0, N * L + 1, L))
    n0 = _core.launch_count()
    pto = KDAChunked("pto", chunk=128)
    o = pto(q, k, v, g, beta, scale=128 ** -0.5, cu_seqlens=cu)
    torch.cuda.synchronize()
    assert _core.launch_count() > n0, "contractions did not run on the native kernels"
    o_t = KDAChunked("torch", chunk=128)(q, k, v, g, beta, scale=128 ** -0.5, cu_seqlens=cu)
    ref = KDAChunked("torch", chunk=128, dtype=torch.float64)(
        *(x.double() for x in (q, k, v, g, beta)), scale=128 ** -0.5, cu_seqlens=cu)
    e_pto, e_torch = rel(o, ref), rel(o_t, ref)
    assert e_pto < 1e-4, (e_pto, e_torch)
    assert e_pto < 10 * e_torch + 1e-6, (e_pto, e_torch)
    pto.cleanup()


@pytest.mark.gpu
def test_kda_graph_replay_matches_eager():
    dev = torch.device("cuda", 0)
    q, k, v, g, beta = random_kda_inputs(512, 4, 2, 128, seed=5, device=dev)
    cu = [0, 256, 512]
    pto = KDAChunked("pto", chunk=128)
    eager = pto(q, k, v, g, beta, cu_seqlens=cu).clone()
    graph = KDAGraph(pto, q, k, v, g, beta, cu_seqlens=cu)
    assert torch.equal(graph(q, k, v, g, beta).clone(), eager)
    q2, k2, v2, g2, b2 = random_kda_inputs(512, 4, 2, 128, seed=6, device=dev)
    assert torch.equal(graph(q2, k2, v2, g2, b2).clone(), pto(q2, k2, v2, g2, b2, cu_seqlens=cu))
    pto.cleanup()
