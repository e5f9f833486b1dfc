"""Chunked gated delta rule (GDN) forward stages on a pluggable two-operand einsum.

The reference exercises its einsum backend with a GDN pipeline whose contraction
stages call one overridable method (benchmarks/complex/gdn/einsum_gdn.py:30-34,
`EinsumGDN._einsum`; benchmarks/complex/gdn/pto_gdn.py:27-39 swaps in pto_einsum
runners cached per (equation, shapes, dtype)). This module is the same kind of caller
for this library: every contraction goes through `self.contract(eq, a, b)`, which is
either torch.einsum (`backend="torch"`) or a cached `EinsumBuilder` runner on the
B200 kernels (`backend="pto"`); the glue (gates, masks, the triangular solve) is torch.

Algorithm: the chunkwise form of the gated delta rule (Yang, Kautz, Hatamizadeh,
"Gated Delta Networks: Improving Mamba2 with Delta Rule", ICLR 2025), state
S in R^{Dk x Dv}, per step t with log-decay g_t and write strength beta_t:

    S_t = exp(g_t) (I - beta_t k_t k_t^T) S_{t-1} + beta_t k_t v_t^T,   o_t = scale * S_t^T q_t.

Per chunk of C steps with in-chunk cumulative log-decay G (G_i = g_1 + ... + g_i):

    A_ij  = beta_i exp(G_i - G_j) k_i.k_j  (j < i)          stage kkt
    T     = (I + A)^-1                                      stage solve_tril
    W     = T (beta exp(G) k),   U = T (beta v)             stage wy_fast
    V'    = U - W S,   S' = exp(G_C) S + K^T (exp(G_C - G) V')   stage chunk_h (sequential)
    O     = exp(G) (Q S) + [(Q K^T) exp(G_i - G_j), j <= i] V'   stage chunk_o

The contraction equations keep the (batch, row, head, feature) layout of the inputs
and let the einsum labels carry the transposes, as the reference's stages do
(einsum_gdn.py:98, :193, :262, :272, :314-323), so the backend sees the same
plans: 'bihd,bjhd->bihj', 'bihj,bjhd->bihd', 'bvhd,bhde->bvhe', 'bvhd,bvhe->bhde'.

B200 specifics: equal-length sequences (cu_seqlens with a common length, or B > 1)
are folded into the batch, so the sequential state pass runs once per chunk index
over all sequences at once instead of once per chunk; the chunk-parallel stages fold
every chunk into the batch (one launch per contraction). `GDNGraph` captures a whole
forward pass for fixed shapes into a CUDA graph so the launch-bound regime of many
small contractions costs one graph launch.
"""
from __future__ import annotations

import torch

__all__ = ["GDNChunked", "GDNGraph", "gdn_recurrent_reference", "random_gdn_inputs"]


def _safe_exp(x: torch.Tensor) -> torch.Tensor:
    # exp of non-positive log-decay differences; positive ones only occur above
    # the diagonal, which the masks remove, and are zeroed so they cannot overflow
    return torch.where(x <= 0, torch.exp(torch.clamp(x, max=0.0)), torch.zeros_like(x))


class GDNChunked:
    """GDN forward stages with a pluggable contraction backend.

    backend: "torch" (torch.einsum) or "pto" (this library's CUDA kernels; one
    EinsumBuilder runner per distinct (equation, shapes, dtype), built on first use
    and reused, as the reference's PtoGDN does).
    """

    def __init__(self, backend: str = "pto", chunk: int = 128, dtype: torch.dtype = torch.float32):
        if backend not in ("torch", "pto"):
            raise ValueError(f"unknown backend {backend!r}")
        self.backend = backend
        self.chunk = chunk
        self.dtype = dtype
        self._runners: dict = {}
        self._builders: list = []

    # -- contraction backend ------------------------------------------------
    def contract(self, eq: str, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        if self.backend == "torch":
            return torch.einsum(eq, a, b)
        from .builder import EinsumBuilder
        a = a.contiguous()
        b = b.contiguous()
        key = (eq, tuple(a.shape), tuple(b.shape), a.dtype)
        run = self._runners.get(key)
        if run is None:
            bld = EinsumBuilder(eq, [tuple(a.shape), tuple(b.shape)], a.dtype)
            run = bld.build()
            self._runners[key] = run
            self._builders.append(bld)
        out = run(a, b)
        return out if out.dtype == self.dtype else out.to(self.dtype)

    def cleanup(self):
        for b in self._builders:
            try:
                b.cleanup()
            except Exception:
                pass
        self._builders.clear()
        self._runners.clear()

    # -- layout ---------------------------------------------------------------
    def fold(self, x: torch.Tensor, cu_seqlens=None) -> torch.Tensor:
        """[B, T, ...] (or [1, total, ...] with equal-length cu_seqlens) -> [N, L, ...]."""
        if cu_seqlens is None:
            L = x.shape[1]
            if L % self.chunk:
                raise ValueError(f"sequence length {L} must be a multiple of the chunk size {self.chunk}")
            return x
        cu = [int(v) for v in (cu_seqlens.tolist() if hasattr(cu_seqlens, "tolist") else cu_seqlens)]
        lens = {cu[i + 1] - cu[i] for i in range(len(cu) - 1)}
        if x.shape[0] != 1 or len(lens) != 1 or cu[0] != 0 or cu[-1] != x.shape[1]:
            raise ValueError("cu_seqlens must split a single batch row into equal-length sequences")
        L = lens.pop()
        if L % self.chunk:
            raise ValueError(f"sequence length {L} must be a multiple of the chunk size {self.chunk}")
        return x.reshape(len(cu) - 1, L, *x.shape[2:])

    def _chunks(self, x: torch.Tensor) -> torch.Tensor:
        """[N, L, ...] -> [N * nc, C, ...] (chunks folded into the batch)."""
        N, L = x.shape[:2]
        return x.reshape(N * (L // self.chunk), self.chunk, *x.shape[2:])

    @staticmethod
    def _expand_heads(x: torch.Tensor, H: int) -> torch.Tensor:
        grp = H // x.shape[2]
        return x if grp == 1 else x.repeat_interleave(grp, dim=2)

    # -- stages (inputs already folded to [N, L, ...]) --------------------------
    def cumsum(self, g: torch.Tensor) -> torch.Tensor:
        N, L, H = g.shape
        gc = g.to(self.dtype).reshape(N, L // self.chunk, self.chunk, H).cumsum(dim=2)
        return gc.reshape(N, L, H)

    def kkt(self, k: torch.Tensor, beta: torch.Tensor, gcum: torch.Tensor) -> torch.Tensor:
        """A[n, i, h, j] = beta_i exp(G_i - G_j) k_i.k_j for j < i, per chunk. Returns [N, L, H, C]."""
        N, L, H = beta.shape
        C = self.chunk
        kc = self._chunks(self._expand_heads(k.to(self.dtype), H))
        gc = self._chunks(gcum)                                   # [Bn, C, H]
        bc = self._chunks(beta.to(self.dtype))
        qk = self.contract("bihd, bjhd -> bihj", kc, kc)          # [Bn, i, H, j]
        decay = _safe_exp(gc.unsqueeze(-1) - gc.permute(0, 2, 1).unsqueeze(1))
        strict = torch.ones(C, C, dtype=torch.bool, device=k.device).tril(-1)
        A = qk * decay * bc.unsqueeze(-1) * strict[None, :, None, :]
        return A.reshape(N, L, H, C)

    def solve_tril(self, A: torch.Tensor) -> torch.Tensor:
        """(I + A)^-1 per chunk and head (A strictly lower). Returns [N, L, H, C]."""
        N, L, H, C = A.shape
        Ab = self._chunks(A).permute(0, 2, 1, 3)                  # [Bn, H, i, j]
        eye = torch.eye(C, dtype=A.dtype, device=A.device).expand_as(Ab)
        inv = torch.linalg.solve_triangular(Ab + eye, eye, upper=False, unitriangular=True)
        return inv.permute(0, 2, 1, 3).reshape(N, L, H, C)

    def wy_fast(self, k, v, beta, Ainv, gcum):
        """W = T (beta exp(G) k), U = T (beta v): one stacked contraction per call."""
        N, L, H = beta.shape
        Dk, Dv = k.shape[-1], v.shape[-1]
        kc = self._chunks(self._expand_heads(k.to(self.dtype), H))
        vc = self._chunks(v.to(self.dtype))
        bc = self._chunks(beta.to(self.dtype)).unsqueeze(-1)
        gc = self._chunks(gcum)
        kb = kc * bc * torch.exp(gc).unsqueeze(-1)
        vb = vc * bc
        rhs = torch.cat([kb, vb], dim=-1)                         # [Bn, j, H, Dk + Dv]
        wu = self.contract("bihj, bjhd -> bihd", self._chunks(Ainv), rhs)
        w = wu[..., :Dk].reshape(N, L, H, Dk)
        u = wu[..., Dk:].reshape(N, L, H, Dv)
        return w, u

    def chunk_h(self, k, w, u, gcum):
        """Sequential state pass, all sequences at once per chunk index.

        Returns (h [N, nc, H, Dk, Dv] = state entering each chunk, v_new [N, L, H, Dv],
        final state [N, H, Dk, Dv])."""
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
            gc = gcum[:, s]                                       # [N, C, H]
            glast = gc[:, -1:]                                    # [N, 1, H]
            vc = u[:, s] - self.contract("bvhd, bhde -> bvhe", w[:, s], S)
            v_new[:, s] = vc
            kv = self.contract("bvhd, bvhe -> bhde", kx[:, s], vc * torch.exp(glast - gc).unsqueeze(-1))
            S = torch.exp(glast).permute(0, 2, 1).unsqueeze(-1) * S + kv
        return h, v_new, S

    def chunk_o(self, q, k, v_new, h, gcum):
        N, L, H, Dv = v_new.shape
        C = self.chunk
        qc = self._chunks(self._expand_heads(q.to(self.dtype), H))
        kc = self._chunks(self._expand_heads(k.to(self.dtype), H))
        vc = self._chunks(v_new)
        gc = self._chunks(gcum)                                   # [Bn, C, H]
        hb = h.reshape(-1, *h.shape[2:])                          # [Bn, H, Dk, Dv]
        inter = self.contract("bvhd, bhde -> bvhe", qc, hb) * torch.exp(gc).unsqueeze(-1)
        qk = self.contract("bihd, bjhd -> bihj", qc, kc)          # [Bn, i, H, j]
        gate = torch.exp(torch.clamp(gc.unsqueeze(-1) - gc.permute(0, 2, 1).unsqueeze(1), max=0.0))
        causal = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
        intra = self.contract("bihj, bjhd -> bihd", qk * gate * causal[None, :, None, :], vc)
        return (inter + intra).reshape(N, L, H, Dv)

    # -- full forward -----------------------------------------------------------
    def forward(self, q, k, v, g, beta, scale: float = 1.0, cu_seqlens=None, return_state: bool = False):
        """q, k [B, T, Hg, Dk]; v [B, T, H, Dv]; g (log-decay), beta [B, T, H].
        Returns o [B, T, H, Dv] (and the final state [N, H, Dk, Dv])."""
        B, T = v.shape[:2]
        if v.shape[2] % k.shape[2]:
            raise ValueError("value heads must be a multiple of key heads")
        f = lambda x: self.fold(x, cu_seqlens)  # noqa: E731
        qf, kf, vf, gf, bf = f(q), f(k), f(v), f(g), f(beta)
        gcum = self.cumsum(gf)
        A = self.kkt(kf, bf, gcum)
        Ainv = self.solve_tril(A)
        w, u = self.wy_fast(kf, vf, bf, Ainv, gcum)
        h, v_new, S = self.chunk_h(kf, w, u, gcum)
        o = self.chunk_o(qf, kf, v_new, h, gcum) * scale
        o = o.reshape(B, T, *o.shape[2:])
        return (o, S) if return_state else o

    __call__ = forward


class GDNGraph:
    """One CUDA graph for a whole GDN forward at fixed shapes.

    The first call (outside capture) builds every runner and its workspace; the
    forward is then captured on a side stream and replayed on later calls after the
    inputs are copied into the graph's static buffers."""

    def __init__(self, gdn: GDNChunked, q, k, v, g, beta, scale: float = 1.0, cu_seqlens=None):
        self.gdn = gdn
        self.scale = scale
        self.cu = cu_seqlens
        self.static = [t.clone() for t in (q, k, v, g, beta)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                gdn.forward(*self.static, scale=scale, cu_seqlens=cu_seqlens)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = gdn.forward(*self.static, scale=scale, cu_seqlens=cu_seqlens)

    def __call__(self, q, k, v, g, beta) -> torch.Tensor:
        for dst, src in zip(self.static, (q, k, v, g, beta)):
            dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.out


def gdn_recurrent_reference(q, k, v, g, beta, scale: float = 1.0):
    """Step-by-step recurrence (float64) for checking the chunked form; small sizes only."""
    B, T, Hg, Dk = q.shape
    H, Dv = v.shape[2], v.shape[3]
    grp = H // Hg
    qd, kd = (x.double().repeat_interleave(grp, dim=2) for x in (q, k))
    vd, gd, bd = v.double(), g.double(), beta.double()
    S = torch.zeros(B, H, Dk, Dv, dtype=torch.float64)
    o = torch.empty(B, T, H, Dv, dtype=torch.float64)
    for t in range(T):
        kt, vt, qt = kd[:, t], vd[:, t], qd[:, t]                   # [B, H, D]
        S = torch.exp(gd[:, t])[..., None, None] * S
        pred = torch.einsum("bhd,bhde->bhe", kt, S)
        S = S + torch.einsum("bhd,bhe->bhde", kt, bd[:, t, :, None] * (vt - pred))
        o[:, t] = torch.einsum("bhd,bhde->bhe", qt, S) * scale
    return o


def random_gdn_inputs(T, H, Hg, D, B=1, seed=0, device="cpu", dtype=torch.float32):
    """Seeded inputs with the usual GDN statistics: unit-norm q and k rows, N(0,1) v,
    beta ~ U[0,1), log-decay g = logsigmoid(N(0,1))."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, T, Hg, D, generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, T, Hg, D, generator=gen), dim=-1)
    v = torch.randn(B, T, H, D, generator=gen)
    beta = torch.rand(B, T, H, generator=gen)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=gen))
    return tuple(x.to(device=device, dtype=dtype) for x in (q, k, v, g, beta))
