"""Equation parser and transpose -> batched-matmul -> transpose planner.

This module restates the planning rules of pto-einsum's ``builder.py`` so that
every equation/shape pair yields the *same* ``EinsumRecipe`` dictionary as the
reference planner (plan identity), field for field:

* ``validate_expr``      follows ``src/pto_einsum/builder.py:148-183``
* ``parse_recipe``       follows ``src/pto_einsum/builder.py:185-367``
* ``try_broadcast``      follows ``src/pto_einsum/builder.py:369-447``
* ``choose_operand_order`` follows ``src/pto_einsum/builder.py:555-604``
* ``tile_k`` / ``splitk_eligible`` follow ``builder.py:463-507`` (these only
  feed the emitted config text; the CUDA backend picks its own tiling)

The recipe is NPU-shaped (fields such as ``in_nt`` describe Ascend read modes)
but it is the contract the code generator consumes, so it is kept bit-for-bit.
The CUDA backend reads the same recipe and lowers it to TMA tensor maps.
"""
from __future__ import annotations

import os
from math import prod
from typing import Optional, Sequence, Tuple, TypedDict

# Broadcast classifier caps. They change which route a plan takes, so they keep
# the reference values (builder.py:20-22).
BCAST_TILECAP = 4096
BCAST_SCALAR_SIZE_CAP = 8192

_LETTERS = frozenset("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ")


def _neutral_broadcast() -> dict:
    return dict(broadcast=False, bc_mode=0, bc_Cc=1, bc_Rr=1, bc_Inner=1, bc_Outer=1,
                bc_sizeB=1, bc_full_is_in0=True, bc_outer_dims=(), bc_outer_bstride=())


def _neutral_fuse() -> dict:
    return dict(out_fusible=0, out_row_stride=0, out_n_batch=0,
                out_batch_sizes=(), out_batch_strides=())


def _neutral_direct() -> dict:
    return dict(in_nt=0, in_n_batch=0, in0_row_stride=0, in0_k_stride=0,
                in1_col_stride=0, in1_k_stride=0, in_batch_sizes=(),
                in0_batch_strides=(), in1_batch_strides=())


class EinsumRecipe(TypedDict):
    """Plan of one two-operand einsum (field meanings: builder.py:44-110)."""
    in_transpose_idxs: Tuple[Tuple[int, ...], Tuple[int, ...]]
    L0: int
    L1: int
    I: int
    C: int
    out_interpret_shape: Tuple[int, ...]
    out_transpose_idxs: Tuple[int, ...]
    out_shape: Tuple[int, ...]
    elementwise: bool
    n_elem: int
    broadcast: bool
    bc_mode: int
    bc_Cc: int
    bc_Rr: int
    bc_Inner: int
    bc_Outer: int
    bc_sizeB: int
    bc_full_is_in0: bool
    bc_outer_dims: tuple
    bc_outer_bstride: tuple
    out_fusible: int
    out_row_stride: int
    out_n_batch: int
    out_batch_sizes: tuple
    out_batch_strides: tuple
    in_nt: int
    in_n_batch: int
    in0_row_stride: int
    in0_k_stride: int
    in1_col_stride: int
    in1_k_stride: int
    in_batch_sizes: tuple
    in0_batch_strides: tuple
    in1_batch_strides: tuple


def tile_size() -> int:
    """Matmul base tile from ``EINSUM_TILE_SIZE`` (default 128, builder.py:319)."""
    return int(os.getenv("EINSUM_TILE_SIZE", "128"))


def _pad16(x: int) -> int:
    return -(-x // 16) * 16


def _c_strides(shape: Sequence[int]) -> list:
    """Row-major element strides of a contiguous tensor."""
    out = [0] * len(shape)
    run = 1
    for p in reversed(range(len(shape))):
        out[p] = run
        run *= int(shape[p])
    return out


def split_equation(fn: str) -> Tuple[str, str, str]:
    """Split ``"a,b->c"`` into stripped subscripts (builder.py:149-150)."""
    parts = fn.split('->')
    if len(parts) != 2:
        raise ValueError(f"einsum string {fn} is invalid: expected exactly one '->'")
    lhs, out = (p.strip() for p in parts)
    ins = lhs.split(',')
    if len(ins) != 2:
        raise ValueError(f"einsum string {fn} is invalid: expected exactly two input operands")
    return ins[0].strip(), ins[1].strip(), out


def validate_expr(fn: str, shape0: Sequence[int], shape1: Sequence[int]):
    """Check subscripts and shapes; return the normalised equation and output shape.

    Same checks, order and messages as ``builder.py:148-183``.
    """
    in0, in1, out = split_equation(fn)
    if not set(in0 + in1 + out) <= _LETTERS:
        raise ValueError(f"einsum string {fn} is invalid: subscripts should be in [a-zA-Z]")
    for label, subs in (("input0", in0), ("input1", in1), ("output", out)):
        seen = set()
        for ch in subs:
            if ch in seen:
                raise ValueError(
                    f"einsum string {fn} is invalid: {label} subscripts includes '{ch}' multiple times")
            seen.add(ch)
    missing = set(out) - set(in0) - set(in1)
    if missing:
        raise ValueError(f'einsum string {fn} is invalid: output subscripts {missing} not found in inputs')
    if len(set(in0)) != len(shape0):
        raise ValueError(f'Input0 requires {len(set(in0))} dimensions, but {len(shape0)} is given')
    if len(set(in1)) != len(shape1):
        raise ValueError(f'Input1 requires {len(set(in1))} dimensions, but {len(shape1)} is given')
    for ch in set(in0) & set(in1):
        d0, d1 = shape0[in0.index(ch)], shape1[in1.index(ch)]
        if d0 != d1:
            raise ValueError(f"Input dimension size mismatches for common subscript '{ch}': {d0} and {d1}")
    sizes = {}
    for ch, d in zip(in1, shape1):
        sizes[ch] = d
    for ch, d in zip(in0, shape0):
        sizes[ch] = d
    out_shape = tuple(sizes[ch] for ch in out)
    return f'{in0},{in1}->{out}', out_shape


def try_broadcast(device: str, in0, in1, out, shape0, shape1, out_shape,
                  extended: bool = False) -> Optional[EinsumRecipe]:
    """Classify a contraction-free equation as a broadcast multiply, else None.

    Mode 0 ("ColExpand"): the broadcast operand B varies along the innermost
    output run; mode 1 ("scalar"): B is constant over the innermost block.
    Follows ``builder.py:369-447``; the CPU device never takes this route.
    ``extended`` drops the reference's tile caps (an inner run above
    BCAST_TILECAP, a scalar-mode operand above BCAST_SCALAR_SIZE_CAP), which it
    sends down the matmul route instead: the CUDA broadcast kernels take any size.
    """
    if device == "cpu":
        return None
    s_out = set(out)
    full_is_in0 = set(in0) == s_out
    full_is_in1 = set(in1) == s_out
    if full_is_in0 == full_is_in1:
        return None
    full, bc = (in0, in1) if full_is_in0 else (in1, in0)
    if list(full) != list(out):
        return None
    n = len(out)
    sizes = [int(s) for s in out_shape]
    pos = [out.index(ch) for ch in bc]
    if pos != sorted(pos):
        return None
    in_b = [out[p] in set(bc) for p in range(n)]
    # strides of B (contiguous in output order) along each output axis, 0 where absent
    bstride = [0] * n
    run = 1
    for p in reversed(range(n)):
        if in_b[p]:
            bstride[p] = run
            run *= sizes[p]
    size_b = prod(sizes[p] for p in pos) if pos else 1

    p = n - 1
    if in_b[n - 1]:
        mode = 0
        cc = 1
        while p >= 0 and in_b[p]:
            if cc * sizes[p] > BCAST_TILECAP and not extended:
                return None
            cc *= sizes[p]
            p -= 1
        rr = 1
        while p >= 0 and not in_b[p]:
            rr *= sizes[p]
            p -= 1
        inner = rr * cc
    else:
        mode = 1
        if size_b > BCAST_SCALAR_SIZE_CAP and not extended:
            return None
        inner = 1
        while p >= 0 and not in_b[p]:
            inner *= sizes[p]
            p -= 1
        cc, rr = 1, 1
    outer_dims = tuple(sizes[q] for q in range(p + 1))
    outer_bstride = tuple(bstride[q] for q in range(p + 1))
    outer = prod(outer_dims) if outer_dims else 1
    recipe = dict(
        in_transpose_idxs=((), ()),
        out_interpret_shape=tuple(out_shape),
        out_transpose_idxs=tuple(range(n)),
        out_shape=tuple(out_shape),
        L0=1, L1=1, I=prod(out_shape), C=1,
        elementwise=False,
        n_elem=prod(out_shape),
        broadcast=True, bc_mode=mode, bc_Cc=cc, bc_Rr=rr, bc_Inner=inner, bc_Outer=outer,
        bc_sizeB=size_b, bc_full_is_in0=full_is_in0,
        bc_outer_dims=outer_dims, bc_outer_bstride=outer_bstride,
    )
    recipe.update(_neutral_fuse())
    recipe.update(_neutral_direct())
    return EinsumRecipe(**recipe)


def parse_recipe(device: str, fn: str, shape0: Sequence[int], shape1: Sequence[int],
                 extended: bool = False) -> EinsumRecipe:
    """Build the plan for one operand order (``builder.py:185-367``); ``extended``
    lifts the broadcast caps (see try_broadcast)."""
    fn, out_shape = validate_expr(fn, shape0, shape1)
    s0, s1, so = split_equation(fn)
    in0, in1, out = list(s0), list(s1), list(so)

    if in0 == in1 == out:
        recipe = dict(
            in_transpose_idxs=((), ()),
            out_interpret_shape=out_shape,
            out_transpose_idxs=tuple(range(len(out_shape))),
            out_shape=out_shape,
            L0=1, L1=1, I=prod(out_shape), C=1,
            elementwise=True,
            n_elem=prod(out_shape),
        )
        recipe.update(_neutral_broadcast())
        recipe.update(_neutral_fuse())
        recipe.update(_neutral_direct())
        return EinsumRecipe(**recipe)

    set0, set1, set_out = set(in0), set(in1), set(out)
    common = set0 & set1
    contracted = common - set_out
    batch = common & set_out

    solo = (set0 - set1 - set_out) | (set1 - set0 - set_out)
    if solo:
        raise ValueError(
            f"einsum '{fn}': index {sorted(solo)} appears in only one operand and "
            "is reduced away; single-operand reduction is not supported.")

    if not contracted:
        bc = try_broadcast(device, in0, in1, out, shape0, shape1, out_shape, extended)
        if bc is not None:
            return bc

    by1 = lambda ch: in1.index(ch)  # noqa: E731
    contract = sorted(contracted, key=by1)
    inplace = sorted(batch, key=by1)
    free0 = sorted((set_out - common) & set0, key=lambda ch: in0.index(ch))
    free1 = sorted((set_out - common) & set1, key=by1)

    perm0 = tuple(in0.index(ch) for ch in inplace + free0 + contract)
    perm1 = tuple(in1.index(ch) for ch in inplace + contract + free1)

    size_of = lambda ch: int(shape0[in0.index(ch)]) if ch in in0 else int(shape1[in1.index(ch)])  # noqa: E731
    inplace_shape = tuple(size_of(ch) for ch in inplace)
    free0_shape = tuple(size_of(ch) for ch in free0)
    free1_shape = tuple(size_of(ch) for ch in free1)
    I = prod(inplace_shape)
    C = prod(size_of(ch) for ch in contract)
    L0, L1 = prod(free0_shape), prod(free1_shape)

    interp_order = inplace + free0 + free1
    out_pos = [out.index(ch) for ch in interp_order]
    # argsort of the output positions: out axis p is interp axis out_perm[p]
    out_perm = tuple(sorted(range(len(out_pos)), key=lambda j: out_pos[j]))
    out_identity = out_perm == tuple(range(len(out_perm)))

    fields = {}
    fused = (len(free0) == 1 and len(free1) == 1
             and out.index(free1[0]) == len(out) - 1 and not out_identity)
    if fused:
        res_st = dict(zip(out, _c_strides(out_shape)))
        fields.update(
            out_fusible=1,
            out_row_stride=int(res_st[free0[0]]),
            out_n_batch=len(inplace),
            out_batch_sizes=tuple(int(s) for s in inplace_shape),
            out_batch_strides=tuple(int(res_st[ch]) for ch in inplace),
        )
    else:
        fields.update(_neutral_fuse())

    single = (os.getenv("EINSUM_DISABLE_NT", "0") == "0"
              and len(contract) == 1 and len(free0) == 1 and len(free1) == 1
              and C % 16 == 0)
    mode = 0
    if single:
        a_k_inner = in0[-1] == contract[0]
        a_m_inner = in0[-1] == free0[0]
        b_n_inner = in1[-1] == free1[0]
        if a_k_inner and in1[-1] == contract[0]:
            mode = 1
        elif a_k_inner and b_n_inner:
            mode = 2
        elif a_m_inner and b_n_inner:
            mode = 3
    if mode:
        t = tile_size()
        mp, np_ = _pad16(L0), _pad16(L1)
        if mp % min(t, mp) or np_ % min(t, np_):
            mode = 0
    if mode:
        st0, st1 = _c_strides(shape0), _c_strides(shape1)
        fields.update(
            in_nt=mode,
            in_n_batch=len(inplace),
            in0_row_stride=int(st0[in0.index(free0[0])]),
            in0_k_stride=int(st0[in0.index(contract[0])]),
            in1_col_stride=int(st1[in1.index(free1[0])]),
            in1_k_stride=int(st1[in1.index(contract[0])]),
            in_batch_sizes=tuple(int(s) for s in inplace_shape),
            in0_batch_strides=tuple(int(st0[in0.index(ch)]) for ch in inplace),
            in1_batch_strides=tuple(int(st1[in1.index(ch)]) for ch in inplace),
        )
    else:
        fields.update(_neutral_direct())

    recipe = dict(
        in_transpose_idxs=(perm0, perm1),
        out_interpret_shape=inplace_shape + free0_shape + free1_shape,
        out_transpose_idxs=out_perm,
        out_shape=out_shape,
        L0=L0, L1=L1, I=I, C=C,
        elementwise=False,
        n_elem=prod(out_shape),
    )
    recipe.update(_neutral_broadcast())
    recipe.update(fields)
    return EinsumRecipe(**recipe)


def is_identity(perm: Sequence[int]) -> bool:
    return tuple(perm) == tuple(range(len(perm)))


def choose_operand_order(device: str, equation: str, shape0, shape1, extended: bool = False):
    """Plan the equation, swapping the operands when that removes an output permute.

    Returns ``(recipe, swapped)``. The swap is adopted only when the natural
    order keeps a non-fusible, non-identity output and the swapped order makes
    it fusible or identity (``builder.py:562-586``).
    """
    recipe = parse_recipe(device, equation, shape0, shape1, extended)
    is_mm = not recipe['elementwise'] and not recipe['broadcast']
    if (os.getenv("EINSUM_DISABLE_OPERAND_SWAP", "0") == "0" and is_mm
            and not recipe['out_fusible'] and not is_identity(recipe['out_transpose_idxs'])):
        a, b, o = split_equation(equation)
        alt = parse_recipe(device, f"{b},{a}->{o}", shape1, shape0, extended)
        if alt['out_fusible'] or is_identity(alt['out_transpose_idxs']):
            return alt, True
    return recipe, False


def partial_tile_message(recipe: EinsumRecipe) -> Optional[str]:
    """Message of the reference's batched partial-tile guard, or None if it passes.

    ``builder.py:588-604`` rejects batched (I>1) plans whose padded free dims are
    not tile multiples. The CUDA backend handles those tiles (TMA zero-fills
    out-of-range rows and clips the store), so the CUDA device does not raise;
    the function is kept so callers can reproduce the reference decision.
    """
    if recipe['I'] <= 1 or recipe['elementwise'] or recipe['broadcast']:
        return None
    t = tile_size()
    L0, L1 = recipe['L0'], recipe['L1']
    mp, np_ = _pad16(L0), _pad16(L1)
    if mp % min(t, mp) == 0 and np_ % min(t, np_) == 0:
        return None
    return (f"batched einsum (I={recipe['I']}) requires each output free dim to be a "
            f"multiple of the matmul tile ({t}) once padded to 16; got "
            f"L0={L0} (Mpad={mp}), L1={L1} (Npad={np_}). Partial tiles are "
            f"currently single-batch (I==1) only.")


def tile_k(dtype_bytes: int, tile: int, L0: int, L1: int, C: int) -> int:
    """NPU K-tile depth (``builder.py:463-486``); emitted into the config text only."""
    mp, np_, kp = _pad16(L0), _pad16(L1), _pad16(C)
    mt, nt = min(tile, mp), min(tile, np_)
    cap = min(65536 // (mt * dtype_bytes), 65536 // (nt * dtype_bytes),
              (512 * 1024) // (2 * (mt + nt) * dtype_bytes), kp)
    cap -= cap % 16
    d = cap
    while d >= 16:
        if kp % d == 0:
            return d
        d -= 16
    return 16


def splitk_eligible(recipe: EinsumRecipe, dtype_bytes: int) -> bool:
    """NPU split-K gate (``builder.py:488-507``); kept for plan reporting only."""
    L0, L1, C, I = recipe['L0'], recipe['L1'], recipe['C'], recipe['I']
    if not is_identity(recipe['out_transpose_idxs']):
        return False
    t = tile_size()
    mp, np_, kp = _pad16(L0), _pad16(L1), _pad16(C)
    mt, nt = min(t, mp), min(t, np_)
    nk = kp // tile_k(dtype_bytes, t, L0, L1, C)
    tiles = I * (-(-mp // mt)) * (-(-np_ // nt))
    return nk >= 2 and tiles < 16


def transpose_config(shape: Sequence[int], perm: Sequence[int]) -> dict:
    """Permute config of one operand (``builder.py:449-461``)."""
    shape = tuple(int(s) for s in shape)
    st = _c_strides(shape)
    return dict(
        dims=len(shape),
        N=prod(shape),
        from_shape=shape,
        to_shape=tuple(shape[p] for p in perm),
        perm=tuple(int(p) for p in perm),
        perm_strides=tuple(int(st[p]) for p in perm),
    )


def axis_groups(equation: str, recipe: EinsumRecipe, swapped: bool) -> Tuple[int, int, int, int]:
    """Axis counts (batch, free0, free1, contract) of a matmul recipe.

    The recipe stores only the group products; the CUDA lowering needs the
    per-group axis counts to build strided tensor maps.
    """
    a, b, o = split_equation(equation)
    if swapped:
        a, b = b, a
    sa, sb, so = set(a), set(b), set(o)
    nb = len(sa & sb & so)
    nc = len((sa & sb) - so)
    n0 = len((so - (sa & sb)) & sa)
    n1 = len((so - (sa & sb)) & sb)
    return nb, n0, n1, nc


def solo_reductions(equation: str):
    """Single-operand reduction labels: (labels only in operand 0 and not in the
    output, same for operand 1). The reference rejects such equations
    (``builder.py:185-367`` via the check above); ``EinsumBuilder(extended=True)``
    computes them by first contracting the owning operand with a ones vector
    over those labels."""
    a, b, o = split_equation(equation.replace(" ", ""))
    sa, sb, so = set(a), set(b), set(o)
    solo0 = [ch for ch in a if ch not in sb and ch not in so]
    solo1 = [ch for ch in b if ch not in sa and ch not in so]
    return solo0, solo1
