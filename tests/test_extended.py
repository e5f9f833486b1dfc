"""Opt-in lifts of the reference's roadmap gaps (EinsumBuilder(extended=True)):
single-operand reduction axes and broadcasts above the reference's tile caps.
The default planner stays identical to the reference (tests/test_planner.py)."""
import pytest
import torch

from pto_einsum import EinsumBuilder, einsum, planner


# ---------------------------------------------------------------------------- CPU: planning
def test_default_still_rejects_single_operand_reduction():
    with pytest.raises(ValueError, match="appears in only one operand"):
        EinsumBuilder("ij,jk->k", [(32, 64), (64, 128)], torch.float32).parse_equation()


@pytest.mark.parametrize("eq,s0,s1,pre,main", [
    ("ij,jk->k", (32, 64), (64, 128), ["ij,i->j"], "j,jk->k"),
    ("ij,jk->j", (32, 64), (64, 128), ["ij,i->j", "jk,k->j"], "j,j->j"),
    ("bij,bjk->bk", (2, 8, 16), (2, 16, 4), ["bij,i->bj"], "bj,bjk->bk"),
    ("abc,cd->ad", (3, 5, 7), (7, 9), ["abc,b->ac"], "ac,cd->ad"),
])
def test_solo_reduction_decomposition(eq, s0, s1, pre, main):
    b = EinsumBuilder(eq, [s0, s1], torch.float16, extended=True)
    b.parse_equation()
    subs, m = b._composite
    assert [s.equation for _, s, _ in subs] == pre
    assert m.equation == main and m.dtype == torch.float32
    assert tuple(b.recipe["out_shape"]) == tuple(torch.einsum(eq, torch.zeros(s0), torch.zeros(s1)).shape)


def test_fully_reduced_operand_rejected():
    with pytest.raises(ValueError, match="reduced to a scalar"):
        EinsumBuilder("i,jk->jk", [(8,), (4, 5)], torch.float32, extended=True).parse_equation()


def test_broadcast_caps_lifted_only_when_extended():
    r, _ = planner.choose_operand_order("cuda", "bsd,d->bsd", (2, 16, 8192), (8192,))
    assert not r["broadcast"]                      # reference: Cc 8192 > 4096 -> matmul route
    r, _ = planner.choose_operand_order("cuda", "bsd,d->bsd", (2, 16, 8192), (8192,), extended=True)
    assert r["broadcast"] and r["bc_mode"] == 0 and r["bc_Cc"] == 8192
    r, _ = planner.choose_operand_order("cuda", "hqk,h->hqk", (16384, 4, 8), (16384,), extended=True)
    assert r["broadcast"] and r["bc_mode"] == 1 and r["bc_sizeB"] == 16384
    assert not planner.choose_operand_order("cuda", "hqk,h->hqk", (16384, 4, 8), (16384,))[0]["broadcast"]


# ---------------------------------------------------------------------------- GPU
SOLO_CASES = [
    ("ij,jk->k", (32, 64), (64, 128)), ("ij,jk->k", (1024, 512), (512, 256)),
    ("ij,jk->j", (32, 64), (64, 128)), ("bij,bjk->bk", (4, 64, 256), (4, 256, 128)),
    ("abc,cd->ad", (3, 500, 70), (70, 90)), ("ijk,kl->il", (64, 3, 300), (300, 40)),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
@pytest.mark.parametrize("eq,s0,s1", SOLO_CASES)
def test_solo_reduction_matches_torch(eq, s0, s1, dtype):
    g = torch.Generator().manual_seed(71)
    a = torch.randn(s0, generator=g).to(dtype)
    b = torch.randn(s1, generator=g).to(dtype)
    out = einsum(eq, a.cuda(), b.cuda(), extended=True)
    assert out.dtype == torch.float32
    exact = torch.einsum(eq, a.double(), b.double())
    scale = torch.einsum(eq, a.double().abs(), b.double().abs())
    assert ((out.cpu().double() - exact).abs() <= 2e-5 * scale + 1e-30).all()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16], ids=["f32", "f16"])
@pytest.mark.parametrize("eq,s0,s1", [
    ("bsd,d->bsd", (2, 16, 8192), (8192,)), ("bsd,sd->bsd", (2, 64, 8192), (64, 8192)),
    ("hqk,h->hqk", (16384, 4, 8), (16384,)),
])
def test_lifted_broadcast_bit_exact(eq, s0, s1, dtype):
    g = torch.Generator().manual_seed(72)
    a = torch.randn(s0, generator=g).to(dtype)
    b = torch.randn(s1, generator=g).to(dtype)
    bld = EinsumBuilder(eq, [s0, s1], dtype, extended=True)
    out = bld.build()(a.cuda(), b.cuda())
    assert bld.recipe["broadcast"]
    # one fp32 product per element: bit-exact against torch in fp32
    assert torch.equal(out.cpu(), torch.einsum(eq, a.float(), b.float()))
    bld.cleanup()
