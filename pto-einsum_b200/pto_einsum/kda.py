"""Chunked Kimi Delta Attention (KDA) forward stages on a pluggable two-operand einsum.

The reference drives its einsum backend with a KDA pipeline the same way as with
GDN: the glue is torch and every two-operand contraction goes through one
overridable method (benchmarks/complex/kda/einsum_kda.py:45-47, swapped for cached
pto_einsum runners in benchmarks/complex/kda/pto_kda.py:25-37). This module is that
caller for this library, sharing the backend, folding and CUDA-graph machinery of
`pto_einsum.gdn`.

Algorithm: the delta rule with a channel-wise forget gate (Kimi Team, "Kimi Linear:
An Expressive, Efficient Attention Architecture", 2025). State S in R^{Dk x Dv};
per step t, per-key-dimension log-decay g_t in R^{Dk} and write strength beta_t:

    S_t = (I - beta_t k_t k_t^T) Diag(exp(g_t)) S_{t-1} + beta_t k_t v_t^T,   o_t = scale * S_t^T q_t.

Per chunk of C steps with the in-chunk cumulative log-decay G_i = g_1 + ... + g_i
(a vector per step), the gate enters the contraction operands element-wise:

    A_ij = beta_i sum_d k_id k_jd exp(G_id - G_jd)   (j < i)                stage kkt
    T    = (I + A)^-1                                                       stage solve_tril
    W    = T (beta exp(G) * k),   U = T (beta v)                            stage wy_fast
    V'   = U - W S,   S' = Diag(exp(G_C)) S + (exp(G_C - G) * k)^T V'        stage chunk_h
    O    = (exp(G) * q) S + [sum_d q_id k_jd exp(G_id - G_jd), j <= i] V'   stage chunk_o

exp(G_i - G_j) is split as exp(G_i - R) * exp(R - G_j) so that kkt and the intra-chunk
part of chunk_o are plain contractions 'bihd,bjhd->bihj' of gated operands; R is the
cumulative decay at the middle of the chunk, which halves the exponent range of each
factor (the identity is exact for any R). The contraction equations are the GDN ones
(einsum_kda.py:7-13): 'bihd,bjhd->bihj', 'bihj,bjhd->bihd', 'bvhd,bhde->bvhe',
'bvhd,bvhe->bhde'.
"""
from __future__ import annotations

import torch

from .gdn import GDNChunked, GDNGraph

__all__ = ["KDAChunked", "KDAGraph", "kda_recurrent_reference", "random_kda_inputs"]


class KDAChunked(GDNChunked):
    """KDA forward stages with a pluggable contraction backend ("torch" or "pto",
    see GDNChunked). Inputs: q, k [B, T, Hk, Dk]; v [B, T, H, Dv]; per-dimension
    log-decay g [B, T, H, Dk]; beta [B, T, H]; H a multiple of Hk."""

    def cumsum(self, g: torch.Tensor) -> torch.Tensor:
        N, L, H, D = g.shape
        gc = g.to(self.dtype).reshape(N, L // self.chunk, self.chunk, H, D).cumsum(dim=2)
        return gc.reshape(N, L, H, D)

    def _split_gate(self, gc: torch.Tensor):
        """exp(G - R), exp(R - G) for chunked G [Bn, C, H, D], R = G at the chunk middle."""
        ref = gc[:, self.chunk // 2 - 1: self.chunk // 2]
        return torch.exp(gc - ref), torch.exp(ref - gc)

    def kkt(self, k: torch.Tensor, beta: torch.Tensor, gcum: torch.Tensor) -> torch.Tensor:
        N, L, H = beta.shape
        C = self.chunk
        kc = self._chunks(self._expand_heads(k.to(self.dtype), H))       # [Bn, C, H, D]
        gc = self._chunks(gcum)
        bc = self._chunks(beta.to(self.dtype))
        up, down = self._split_gate(gc)
        A = self.contract("bihd, bjhd -> bihj", kc * up, kc * down)     # [Bn, i, H, j]
        strict = torch.ones(C, C, dtype=torch.bool, device=k.device).tril(-1)
        A = A * bc.unsqueeze(-1) * strict[None, :, None, :]
        return A.reshape(N, L, H, C)

    def wy_fast(self, k, v, beta, Ainv, gcum):
        N, L, H = beta.shape
        Dk, Dv = k.shape[-1], v.shape[-1]
        kc = self._chunks(self._expand_heads(k.to(self.dtype), H))
        vc = self._chunks(v.to(self.dtype))
        bc = self._chunks(beta.to(self.dtype)).unsqueeze(-1)
        gc = self._chunks(gcum)
        rhs = torch.cat([kc * torch.exp(gc) * bc, vc * bc], dim=-1)     # [Bn, j, H, Dk + Dv]
        wu = self.contract("bihj, bjhd -> bihd", self._chunks(Ainv), rhs)
        return wu[..., :Dk].reshape(N, L, H, Dk), wu[..., Dk:].reshape(N, L, H, Dv)

    def chunk_h(self, k, w, u, gcum):
        N, L, H, Dk = w.shape
        Dv = u.shape[-1]
        C = self.chunk
        nc = L // C
        kx = self._expand_heads(k.to(self.dtype), H)
        S = torch.zeros(N, H, Dk, Dv, dtype=self.dtype, device=w.device)
        h = torch.empty(N, nc, H, Dk, Dv, dtype=self.dtype, device=w.device)
        v_new = torch.empty(N, L, H, Dv, dtype=self.dtype, device=w.device)
        for c in range(nc):
            s = slice(c * C, (c + 1) * C)
            h[:, c] = S
            gc = gcum[:, s]                                            # [N, C, H, Dk]
            glast = gc[:, -1:]                                         # [N, 1, H, Dk]
            vc = u[:, s] - self.contract("bvhd, bhde -> bvhe", w[:, s], S)
            v_new[:, s] = vc
            kv = self.contract("bvhd, bvhe -> bhde", kx[:, s] * torch.exp(glast - gc), vc)
            S = torch.exp(glast[:, 0]).unsqueeze(-1) * S + kv           # rows scaled per key dim
        return h, v_new, S

    def chunk_o(self, q, k, v_new, h, gcum):
        N, L, H, Dv = v_new.shape
        C = self.chunk
        qc = self._chunks(self._expand_heads(q.to(self.dtype), H))
        kc = self._chunks(self._expand_heads(k.to(self.dtype), H))
        vc = self._chunks(v_new)
        gc = self._chunks(gcum)
        hb = h.reshape(-1, *h.shape[2:])                               # [Bn, H, Dk, Dv]
        inter = self.contract("bvhd, bhde -> bvhe", qc * torch.exp(gc), hb)
        up, down = self._split_gate(gc)
        qk = self.contract("bihd, bjhd -> bihj", qc * up, kc * down)  # [Bn, i, H, j]
        causal = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
        intra = self.contract("bihj, bjhd -> bihd", qk * causal[None, :, None, :], vc)
        return (inter + intra).reshape(N, L, H, Dv)

    def forward(self, q, k, v, g, beta, scale: float = 1.0, cu_seqlens=None, return_state: bool = False):
        if g.dim() != 4 or g.shape[-1] != k.shape[-1]:
            raise ValueError("KDA gate g must be [B, T, H, Dk] (one log-decay per key dimension)")
        return super().forward(q, k, v, g, beta, scale=scale, cu_seqlens=cu_seqlens, return_state=return_state)

    __call__ = forward


class KDAGraph(GDNGraph):
    """One CUDA graph for a whole KDA forward at fixed shapes (see GDNGraph)."""


def kda_recurrent_reference(q, k, v, g, beta, scale: float = 1.0):
    """Step-by-step KDA recurrence in float64; small sizes only."""
    B, T, Hk, Dk = q.shape
    H, Dv = v.shape[2], v.shape[3]
    grp = H // Hk
    qd, kd = (x.double().repeat_interleave(grp, dim=2) for x in (q, k))
    vd, gd, bd = v.double(), g.double(), beta.double()
    S = torch.zeros(B, H, Dk, Dv, dtype=torch.float64)
    o = torch.empty(B, T, H, Dv, dtype=torch.float64)
    for t in range(T):
        kt, vt, qt = kd[:, t], vd[:, t], qd[:, t]                      # [B, H, D]
        S = torch.exp(gd[:, t]).unsqueeze(-1) * S                      # Diag(alpha_t) S
        pred = torch.einsum("bhd,bhde->bhe", kt, S)
        S = S + torch.einsum("bhd,bhe->bhde", kt, bd[:, t, :, None] * (vt - pred))
        o[:, t] = torch.einsum("bhd,bhde->bhe", qt, S) * scale
    return o


def random_kda_inputs(T, H, Hk, D, B=1, seed=0, device="cpu", dtype=torch.float32, gate=0.05):
    """Seeded KDA inputs: unit-norm q and k rows, N(0,1) v, beta = sigmoid(N(0,1)),
    per-dimension log-decay g ~ U(-gate, 0] (the reference's benchmark draws it in
    (-0.05, 0), benchmarks/complex/kda/utils.py:48-70)."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, generator=gen), dim=-1)
    v = torch.randn(B, T, H, D, generator=gen)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    g = -torch.rand(B, T, H, D, generator=gen) * gate
    return tuple(x.to(device=device, dtype=dtype) for x in (q, k, v, g, beta))
