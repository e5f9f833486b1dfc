"""GDN caller (pto_einsum.gdn): the chunked stages against the step recurrence (CPU),
the B200 contraction backend against torch.einsum and float64 (GPU), CUDA-graph
replay. Mirrors the reference's GDN checks (benchmarks/complex/gdn/
test_gdn_e2e.py, test_gdn_single_kernels.py: Frobenius-relative error of the
pipeline against a float reference, tolerance utils.py:8-14 ftol 1e-3)."""
import pytest
import torch

from pto_einsum import _core
from pto_einsum.gdn import GDNChunked, GDNGraph, gdn_recurrent_reference, random_gdn_inputs


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm()).item()


@pytest.mark.parametrize("B,T,H,Hg,D,C", [(1, 96, 2, 2, 8, 32), (2, 128, 4, 2, 16, 32), (1, 64, 3, 1, 8, 16)])
def test_chunked_matches_recurrence_fp64(B, T, H, Hg, D, C):
    q, k, v, g, beta = random_gdn_inputs(T, H, Hg, D, B=B, seed=T + H, dtype=torch.float64)
    o = GDNChunked("torch", chunk=C, dtype=torch.float64)(q, k, v, g, beta, scale=D ** -0.5)
    r = gdn_recurrent_reference(q, k, v, g, beta, scale=D ** -0.5)
    assert rel(o, r) < 1e-12


def test_chunked_fp32_and_final_state():
    q, k, v, g, beta = random_gdn_inputs(128, 4, 2, 16, B=1, seed=7)
    m = GDNChunked("torch", chunk=32)
    o, S = m(q, k, v, g, beta, return_state=True)
    r = gdn_recurrent_reference(q, k, v, g, beta)
    assert rel(o, r) < 1e-5
    # final state from the recurrence: replay it once more and compare
    q64, k64, v64, g64, b64 = (x.double() for x in (q, k, v, g, beta))
    S64 = torch.zeros(1, 4, 16, 16, dtype=torch.float64)
    kx = k64.repeat_interleave(2, dim=2)
    for t in range(128):
        S64 = torch.exp(g64[:, t])[..., None, None] * S64
        pred = torch.einsum("bhd,bhde->bhe", kx[:, t], S64)
        S64 = S64 + torch.einsum("bhd,bhe->bhde", kx[:, t], b64[:, t, :, None] * (v64[:, t] - pred))
    assert rel(S, S64) < 1e-5


def test_equal_length_sequences_fold():
    q, k, v, g, beta = random_gdn_inputs(64, 2, 2, 8, B=3, seed=11, dtype=torch.float64)
    m = GDNChunked("torch", chunk=16, dtype=torch.float64)
    o = m(q, k, v, g, beta)
    flat = [x.reshape(1, 192, *x.shape[2:]) for x in (q, k, v, g, beta)]
    o1 = m(*flat, cu_seqlens=[0, 64, 128, 192])
    assert rel(o1.reshape(o.shape), o) == 0.0


def test_layout_errors():
    q, k, v, g, beta = random_gdn_inputs(96, 2, 2, 8, seed=1)
    m = GDNChunked("torch", chunk=64)
    with pytest.raises(ValueError, match="multiple of the chunk size"):
        m(q, k, v, g, beta)
    flat = [x.reshape(1, 96, *x.shape[2:]) for x in (q, k, v, g, beta)]
    with pytest.raises(ValueError, match="equal-length"):
        GDNChunked("torch", chunk=32)(*flat, cu_seqlens=[0, 32, 96])
    with pytest.raises(ValueError):
        GDNChunked("cublas")


# ---------------------------------------------------------------------------- GPU
GPU_CASES = [  # (N_seq, L_seg, H, Hg): chunk 128, head dim 128, like the reference's 4-way bench
    (1, 256, 4, 2), (2, 256, 4, 4), (1, 512, 8, 4),
]


@pytest.mark.gpu
@pytest.mark.parametrize("N,L,H,Hg", GPU_CASES)
def test_pto_backend_matches_torch_and_fp64(N, L, H, Hg):
    dev = torch.device("cuda", 0)
    q, k, v, g, beta = random_gdn_inputs(N * L, H, Hg, 128, seed=N * L + H, device=dev)
    cu = list(range(0, N * L + 1, L))
    n0 = _core.core_lib().pe_launch_count()
    pto = GDNChunked("pto", chunk=128)
    o = pto(q, k, v, g, beta, scale=128 ** -0.5, cu_seqlens=cu)
    torch.cuda.synchronize()
    assert _core.core_lib().pe_launch_count() > n0, "contractions did not run on the native kernels"
    o_t = GDNChunked("torch", chunk=128)(q, k, v, g, beta, scale=128 ** -0.5, cu_seqlens=cu)
    ref = GDNChunked("torch", chunk=128, dtype=torch.float64)(
        *(x.double() for x in (q, k, v, g, beta)), scale=128 ** -0.5, cu_seqlens=cu)
    e_pto, e_torch = rel(o, ref), rel(o_t, ref)
    # 3xTF32 contractions: as accurate as fp32; the reference's GDN tolerance is 1e-3
    assert e_pto < 1e-4, (e_pto, e_torch)
    assert e_pto < 10 * e_torch + 1e-6, (e_pto, e_torch)
    pto.cleanup()


@pytest.mark.gpu
def test_gdn_graph_replay_matches_eager():
    dev = torch.device("cuda", 0)
    q, k, v, g, beta = random_gdn_inputs(512, 4, 2, 128, seed=5, device=dev)
    cu = [0, 256, 512]
    pto = GDNChunked("pto", chunk=128)
    eager = pto(q, k, v, g, beta, cu_seqlens=cu).clone()
    graph = GDNGraph(pto, q, k, v, g, beta, cu_seqlens=cu)
    out = graph(q, k, v, g, beta).clone()
    assert torch.equal(out, eager)
    # new inputs through the same graph
    q2, k2, v2, g2, b2 = random_gdn_inputs(512, 4, 2, 128, seed=6, device=dev)
    out2 = graph(q2, k2, v2, g2, b2).clone()
    assert torch.equal(out2, pto(q2, k2, v2, g2, b2, cu_seqlens=cu))
    pto.cleanup()
