"""EinsumBuilder / einsum: plan, generate, compile, cache and run on B200.

Public surface and behaviour follow the reference ``src/pto_einsum/builder.py``:

* ``EinsumBuilder(equation, input_shapes, dtype, device)`` with
  ``parse_equation`` (:555-604), ``generate_code`` (:606-683), ``compile``
  (:685-736), ``load_library`` (:761-815), ``build`` (:817-884),
  ``cleanup`` (:748-759) and the ``recipe`` / ``cpp_code`` / ``so_filename`` /
  ``target_dir`` / ``code_hash`` attributes;
* ``einsum(equation, a, b, device=...)`` (:887-902);
* the md5-keyed on-disk cache ``$EINSUM_BUILD_DIR/<md5>/einsum_<md5>[_tag].{cpp,so}``.

Differences, all deliberate:

* the accelerator backend is CUDA (sm_100a). ``device`` is ``"cuda"``,
  ``"cuda:N"`` or a ``torch.device``; ``"npu"`` is accepted as an alias of the
  current CUDA device so reference call sites run unchanged.
* ``device="cpu"`` plans with the reference's CPU semantics (no broadcast
  route) and runs a host library generated from ``include/pto_einsum_cpu.h``
  (g++, no FMA contraction, host threads), bit-identical to the reference CPU
  path (:606-626, :704-709, :856-875); float16 is rejected there as in the
  reference.
* the generated library is a g++-compiled C++ shim that forwards to the
  prebuilt core library, so a cache miss costs ~0.3 s instead of an nvcc run.
* the batched partial-tile guard (:588-604) is not raised: the CUDA kernels
  handle partial tiles in every batch (TMA zero-fill on load, clipped stores).
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import shutil
import subprocess
from math import prod
from typing import Sequence

import torch

from . import planner, templates
from ._core import INCLUDE_DIR, LIB_DIR, PE_F16, PE_F32, core_lib, core_version, error_string
from .planner import EinsumRecipe

__all__ = ["EinsumBuilder", "einsum", "INCLUDE_DIR", "EinsumRecipe"]


def _cuda_device(device) -> torch.device:
    if isinstance(device, torch.device):
        dev = device
    else:
        s = str(device)
        if s == "npu" or s.startswith("npu:"):
            s = "cuda" + s[3:]
        dev = torch.device(s)
    if dev.type != "cuda":
        raise ValueError(f"pto_einsum runs on CUDA devices; got device={device!r}")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


def _raw_stream_getter():
    """Function device index -> current CUDA stream handle (int). torch's own
    accessor avoids building a Stream object per call where it exists."""
    f = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if f is not None:
        return f
    return lambda idx: torch.cuda.current_stream(idx).cuda_stream


class EinsumBuilder:
    """Plan, compile (with caching) and run one two-operand einsum on a B200."""

    def __init__(self, equation: str, input_shapes: Sequence[Sequence[int]], dtype: torch.dtype,
                 device="cuda", extended: bool = False):
        """``extended=False`` plans exactly as the reference. ``extended=True`` lifts
        two of the reference's roadmap gaps (IMPLEMENTATION.md "Roadmap"): broadcasts
        whose inner run exceeds its tile cap stay broadcasts instead of taking the
        matmul route, and single-operand reduction axes (``ij,jk->k``), which the
        reference rejects, are summed by a first contraction of the owning operand
        with a ones vector; the remaining einsum then runs in fp32."""
        self.equation = equation
        self.extended = extended
        self._composite = None          # (pre-reductions, main builder) for solo axes
        self.input_shapes = input_shapes
        self.dtype = dtype
        self.device = device
        self.include_dir = INCLUDE_DIR
        base = os.getenv("EINSUM_BUILD_DIR")
        self.build_base = os.path.abspath(base) if base else os.path.join(os.getcwd(), "build")
        self.recipe = None
        self.cpp_code = None
        self.cpp_filename = None
        self.so_filename = None
        self.lib = None
        self.c_type = None
        self.code_hash = None
        self.target_dir = None
        self._workspace = None          # {device index: workspace handle}
        self._splitk = False
        self._swap_operands = False
        self._exec_shapes = tuple(input_shapes)
        self._axes = None

    # ---- planning (device-aware exactly like the reference) ----------------
    @property
    def _plan_device(self) -> str:
        return "cpu" if str(self.device) == "cpu" else "cuda"

    def _validate_einsum_expr(self, fn, shape0, shape1):
        return planner.validate_expr(fn, shape0, shape1)

    def parse_recipe(self, fn, input_shape0, input_shape1) -> EinsumRecipe:
        return planner.parse_recipe(self._plan_device, fn, input_shape0, input_shape1)

    def _try_broadcast(self, in0, in1, out, shape0, shape1, out_shape):
        return planner.try_broadcast(self._plan_device, in0, in1, out, shape0, shape1, out_shape)

    def transpose_config_gen(self, name, shape, perm):
        cfg = planner.transpose_config(shape, perm)
        j = lambda xs: ', '.join(str(int(x)) for x in xs)  # noqa: E731
        return dict(dims=cfg['dims'], N=cfg['N'], from_shape=j(cfg['from_shape']), perm=j(cfg['perm']),
                    perm_strides=j(cfg['perm_strides']), to_shape=j(cfg['to_shape']), config_name=name)

    def _dtype_bytes(self) -> int:
        return 2 if self.dtype in (torch.float16, torch.bfloat16) else 4

    def _tile_k(self, tile, L0, L1, C):
        return planner.tile_k(self._dtype_bytes(), tile, L0, L1, C)

    def _splitk_eligible(self) -> bool:
        return planner.splitk_eligible(self.recipe, self._dtype_bytes())

    def parse_equation(self):
        if len(self.input_shapes) != 2:
            raise ValueError("Only exactly two input shapes are supported.")
        shape0, shape1 = (tuple(int(d) for d in s) for s in self.input_shapes)
        if self.extended and self._plan_solo_reductions(shape0, shape1):
            return
        self.recipe, self._swap_operands = planner.choose_operand_order(
            self._plan_device, self.equation, shape0, shape1, self.extended)
        self._exec_shapes = (shape1, shape0) if self._swap_operands else (shape0, shape1)
        r = self.recipe
        if not r['elementwise'] and not r['broadcast']:
            self._axes = planner.axis_groups(self.equation, r, self._swap_operands)

    def _plan_solo_reductions(self, shape0, shape1) -> bool:
        """Split an equation with single-operand reduction axes into per-operand
        pre-contractions with ones vectors plus the remaining two-operand einsum.
        Returns False when the equation has no such axes."""
        solo = planner.solo_reductions(self.equation)
        if not solo[0] and not solo[1]:
            return False
        planner.validate_expr(self.equation, shape0, shape1)
        a, b, o = planner.split_equation(self.equation.replace(" ", ""))
        pre = []
        labels, shapes = [], []
        for k, (lab, shp, sol) in enumerate(((a, shape0, solo[0]), (b, shape1, solo[1]))):
            kept = "".join(ch for ch in lab if ch not in sol)
            if sol:
                if not kept:
                    raise ValueError(f"einsum '{self.equation}': operand {k} is reduced to a scalar; "
                                     "at least one of its indices must remain")
                ones_shape = tuple(shp[lab.index(ch)] for ch in sol)
                sub = EinsumBuilder(f"{lab},{''.join(sol)}->{kept}", [shp, ones_shape], self.dtype,
                                    device=self.device)
                sub.parse_equation()
                pre.append((k, sub, ones_shape))
                shp = tuple(shp[lab.index(ch)] for ch in kept)
            labels.append(kept)
            shapes.append(tuple(shp))
        main = EinsumBuilder(f"{labels[0]},{labels[1]}->{o}", shapes, torch.float32, device=self.device,
                             extended=True)
        main.parse_equation()
        self._composite = (pre, main)
        self.recipe = main.recipe
        self._swap_operands = False
        return True

    def _build_composite(self):
        pre, main = self._composite
        runs = [(k, sub.build(), ones_shape) for k, sub, ones_shape in pre]
        main_run = main.build()
        ones = {}
        shapes = (tuple(self.input_shapes[0]), tuple(self.input_shapes[1]))

        def run(*operands):
            if len(operands) != 2:
                raise ValueError("Expected exactly two operands.")
            ops = list(operands)
            for k in (0, 1):
                if tuple(ops[k].shape) != shapes[k]:
                    raise ValueError(f"Input shapes {ops[0].shape} and {ops[1].shape} do not match built "
                                     f"shapes {self.input_shapes}.")
                if ops[k].dtype != self.dtype:
                    raise TypeError(f"Input datatypes {ops[0].dtype} and {ops[1].dtype} do not match built "
                                    f"datatype {self.dtype}.")
            for k, sub_run, ones_shape in runs:
                key = (k, ops[k].device)
                if key not in ones:
                    ones[key] = torch.ones(ones_shape, dtype=self.dtype, device=ops[k].device)
                ops[k] = sub_run(ops[k], ones[key])
            ops = [x if x.dtype == torch.float32 else x.float() for x in ops]
            return main_run(ops[0], ops[1])

        return run

    def einsum_config_gen(self, tpose_inp0_name, tpose_inp1_name, tpose_out_name):
        r = self.recipe
        tile = planner.tile_size()
        j = lambda xs: ', '.join(str(int(x)) for x in (xs or (0,)))  # noqa: E731
        nb, n0, n1, nc = self._axes
        return dict(
            tpose_inp0_name=tpose_inp0_name, tpose_inp1_name=tpose_inp1_name, tpose_out_name=tpose_out_name,
            n_free0=r['L0'], n_free1=r['L1'], n_contract=r['C'], n_inplace=r['I'],
            tile_m=tile, tile_n=tile, tile_k=self._tile_k(tile, r['L0'], r['L1'], r['C']),
            out_fusible=r['out_fusible'], out_row_stride=r['out_row_stride'], out_n_batch=r['out_n_batch'],
            NB=max(1, len(r['out_batch_sizes'])), out_batch_sizes=j(r['out_batch_sizes']),
            out_batch_strides=j(r['out_batch_strides']),
            in_nt=r['in_nt'], in_n_batch=r['in_n_batch'], in0_row_stride=r['in0_row_stride'],
            in0_k_stride=r['in0_k_stride'], in1_col_stride=r['in1_col_stride'], in1_k_stride=r['in1_k_stride'],
            NIB=max(1, len(r['in_batch_sizes'])), in_batch_sizes=j(r['in_batch_sizes']),
            in0_batch_strides=j(r['in0_batch_strides']), in1_batch_strides=j(r['in1_batch_strides']),
            n_batch=nb, n_free0_axes=n0, n_free1_axes=n1, n_contract_axes=nc,
        )

    # ---- code generation ------------------------------------------------------
    def generate_code(self):
        on_cpu = self._plan_device == "cpu"
        if self.dtype == torch.float32:
            data_t, self.c_type, pe_dtype = 'float', ctypes.c_float, PE_F32
        elif self.dtype == torch.float16:
            if on_cpu:
                raise TypeError("float16 is not supported on CPU")
            data_t, self.c_type, pe_dtype = 'half', ctypes.c_uint16, PE_F16
        else:
            raise TypeError(f"Unsupported torch dtype: {self.dtype}")
        if self.recipe is None:
            self.parse_equation()
        r = self.recipe
        if on_cpu:
            self._generate_cpu_code(data_t)
            return
        prelude = templates.PRELUDE.format(
            equation=self.equation.replace('\n', ' '), shapes=[tuple(s) for s in self.input_shapes],
            dtype=str(self.dtype), core=core_version(), pe_dtype=pe_dtype)
        if r['elementwise']:
            cfg = templates.ELEMENTWISE_CONFIG.format(N=r['n_elem'])
            code = templates.ELEMENTWISE_LIB.format(prelude=prelude, config_code=cfg, data_t=data_t)
        elif r['broadcast']:
            dims = r['bc_outer_dims'] or (1,)
            bst = r['bc_outer_bstride'] or (0,)
            cfg = templates.BROADCAST_CONFIG.format(
                mode=r['bc_mode'], N=r['n_elem'], Cc=r['bc_Cc'], Rr=r['bc_Rr'], Inner=r['bc_Inner'],
                Outer=r['bc_Outer'], sizeB=r['bc_sizeB'], outer_rank=len(r['bc_outer_dims']),
                OR=max(1, len(r['bc_outer_dims'])), outer_dims=', '.join(map(str, dims)),
                outer_bstride=', '.join(map(str, bst)))
            full, bcast = ('input0', 'input1') if r['bc_full_is_in0'] else ('input1', 'input0')
            code = templates.BROADCAST_LIB.format(prelude=prelude, config_code=cfg, data_t=data_t,
                                                  full=full, bcast=bcast)
        else:
            shape0, shape1 = self._exec_shapes
            names = ('config_tpose_inp0', 'config_tpose_inp1', 'config_tpose_out')
            t0 = templates.PERMUTE_CONFIG.format(**self.transpose_config_gen(names[0], shape0, r['in_transpose_idxs'][0]))
            t1 = templates.PERMUTE_CONFIG.format(**self.transpose_config_gen(names[1], shape1, r['in_transpose_idxs'][1]))
            to = templates.PERMUTE_CONFIG.format(**self.transpose_config_gen(
                names[2], r['out_interpret_shape'], r['out_transpose_idxs']))
            ec = templates.EINSUM_CONFIG.format(**self.einsum_config_gen(*names))
            code = templates.MATMUL_LIB.format(
                prelude=prelude, tpose_inp0_code=t0, tpose_inp1_code=t1, tpose_out_code=to, einsum_code=ec,
                data_t=data_t, tpose_inp0_name=names[0], tpose_inp1_name=names[1], tpose_out_name=names[2])
        self.cpp_code = code
        self.code_hash = hashlib.md5(code.encode('utf-8')).hexdigest()
        self.target_dir = os.path.join(self.build_base, self.code_hash)

    def _generate_cpu_code(self, data_t):
        """device="cpu": a host library computing with pto_einsum_cpu.h, bit-identical
        to the reference CPU path (on CPU the planner never takes the broadcast route,
        builder.py:373-376 of the reference)."""
        r = self.recipe
        prelude = templates.CPU_PRELUDE.format(
            equation=self.equation.replace('\n', ' '), shapes=[tuple(s) for s in self.input_shapes],
            dtype=str(self.dtype))
        if r['elementwise']:
            cfg = templates.ELEMENTWISE_CONFIG.format(N=r['n_elem'])
            code = templates.CPU_ELEMENTWISE_LIB.format(prelude=prelude, config_code=cfg, data_t=data_t)
        else:
            shape0, shape1 = self._exec_shapes
            names = ('config_tpose_inp0', 'config_tpose_inp1', 'config_tpose_out')
            t0 = templates.PERMUTE_CONFIG.format(**self.transpose_config_gen(names[0], shape0, r['in_transpose_idxs'][0]))
            t1 = templates.PERMUTE_CONFIG.format(**self.transpose_config_gen(names[1], shape1, r['in_transpose_idxs'][1]))
            to = templates.PERMUTE_CONFIG.format(**self.transpose_config_gen(
                names[2], r['out_interpret_shape'], r['out_transpose_idxs']))
            ec = templates.EINSUM_CONFIG.format(**self.einsum_config_gen(*names))
            code = templates.CPU_MATMUL_LIB.format(prelude=prelude, tpose_inp0_code=t0, tpose_inp1_code=t1,
                                                   tpose_out_code=to, einsum_code=ec, data_t=data_t)
        self.cpp_code = code
        self.code_hash = hashlib.md5(code.encode('utf-8')).hexdigest()
        self.target_dir = os.path.join(self.build_base, self.code_hash)

    def compile(self):
        os.makedirs(self.target_dir, exist_ok=True)
        extra = os.environ.get("EINSUM_EXTRA_DEFINES", "").split()
        tag = "_" + hashlib.md5(" ".join(extra).encode()).hexdigest()[:8] if extra else ""
        self.cpp_filename = os.path.join(self.target_dir, f"einsum_{self.code_hash}{tag}.cpp")
        self.so_filename = os.path.join(self.target_dir, f"einsum_{self.code_hash}{tag}.so")
        if os.path.exists(self.so_filename):
            return
        with open(self.cpp_filename, 'w') as f:
            f.write(self.cpp_code)
        cxx = os.environ.get("CXX", "g++")
        tmp = f"{self.so_filename}.{os.getpid()}.tmp"
        if self._plan_device == "cpu":
            # no FMA contraction: every product and sum rounds once, as on the reference
            cmd = [cxx, "-O3", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC", "-std=c++17",
                   "-pthread", "-I", self.include_dir, *extra, self.cpp_filename, "-o", tmp]
        else:
            cmd = [cxx, "-O2", "-shared", "-fPIC", "-std=c++17", "-I", self.include_dir, *extra,
                   self.cpp_filename, "-o", tmp, "-L", LIB_DIR, "-lpto_einsum_b200",
                   f"-Wl,-rpath,{LIB_DIR}"]
        try:
            res = subprocess.run(cmd, capture_output=True, text=True)
        except OSError as e:
            raise RuntimeError(f"Compilation failed: cannot run the compiler {cxx!r} ({e}); set CXX to a "
                               "working C++17 compiler") from e
        if res.returncode != 0:
            raise RuntimeError(f"Compilation failed:\n{res.stderr}")
        os.replace(tmp, self.so_filename)  # atomic: concurrent builders never see a partial .so

    def load_library(self):
        P = ctypes.POINTER
        T = self.c_type
        fp = P(ctypes.c_float)
        r = self.recipe
        if self._plan_device == "cpu":
            # host library: run_einsum only (synchronous), like the reference's CPU .so
            self.lib = ctypes.CDLL(self.so_filename)
            self.lib.run_einsum.argtypes = [ctypes.c_void_p] * 4
            self.lib.run_einsum.restype = None
            self.lib.run_einsum_last_error.argtypes = []
            self.lib.run_einsum_last_error.restype = ctypes.c_int
            return
        core_lib()  # the shim resolves its pe_* symbols against the core library
        self.lib = ctypes.CDLL(self.so_filename)
        if not r['elementwise'] and not r['broadcast']:
            for name in ('run_transpose_inp0', 'run_transpose_inp1'):
                fn = getattr(self.lib, name)
                fn.argtypes = [P(T), P(T), ctypes.c_void_p]
                fn.restype = None
            self.lib.run_transpose_out.argtypes = [fp, fp, ctypes.c_void_p]
            self.lib.run_transpose_out.restype = None
            self.lib.run_batched_matmul.argtypes = [P(T), P(T), fp, ctypes.c_void_p]
            self.lib.run_batched_matmul.restype = None
        self.lib.run_einsum.argtypes = [P(T), P(T), fp, ctypes.c_void_p]
        self.lib.run_einsum.restype = None
        self.lib.run_einsum_setup.argtypes = [ctypes.c_void_p]
        self.lib.run_einsum_setup.restype = ctypes.c_void_p
        # exec is the per-call hot path: plain addresses (ints) avoid building
        # ctypes pointer objects on every call; pointer instances are accepted too
        self.lib.run_einsum_exec.argtypes = [ctypes.c_void_p] * 5
        self.lib.run_einsum_exec.restype = None
        # same call returning its status (one foreign call per runner call)
        self.lib.run_einsum_exec_rc.argtypes = [ctypes.c_void_p] * 5
        self.lib.run_einsum_exec_rc.restype = ctypes.c_int
        self.lib.run_einsum_teardown.argtypes = [ctypes.c_void_p]
        self.lib.run_einsum_teardown.restype = None
        self.lib.run_einsum_last_error.argtypes = []
        self.lib.run_einsum_last_error.restype = ctypes.c_int

    def _check(self, what: str):
        rc = self.lib.run_einsum_last_error()
        if rc:
            raise RuntimeError(f"pto_einsum: {what} failed for '{self.equation}': {error_string(rc)} ({rc})")

    def _ptr(self, t, ctype):
        return ctypes.cast(t.data_ptr(), ctypes.POINTER(ctype))

    def workspace(self, dev: torch.device, stream_ptr: int):
        """Persistent workspace for `dev` (allocated on first use, like einsum_setup)."""
        if self._workspace is None:
            self._workspace = {}
        ws = self._workspace.get(dev.index)
        if ws is None:
            with torch.cuda.device(dev):
                ws = self.lib.run_einsum_setup(ctypes.c_void_p(stream_ptr))
            if self.lib.run_einsum_last_error():
                self.lib.run_einsum_teardown(ctypes.c_void_p(ws))
                self._check("run_einsum_setup")
            self._workspace[dev.index] = ws
        return ws

    def build(self):
        self.parse_equation()
        if self._composite is not None:
            return self._build_composite()
        self.generate_code()
        self.compile()
        try:
            self.load_library()
        except OSError:
            # a damaged cache entry (truncated or overwritten .so): rebuild it once;
            # a second failure is raised
            os.remove(self.so_filename)
            self.compile()
            self.load_library()
        r = self.recipe
        self._splitk = False if (r['elementwise'] or r['broadcast']) else self._splitk_eligible()
        out_shape = tuple(r['out_shape'])

        shapes = (tuple(self.input_shapes[0]), tuple(self.input_shapes[1]))
        dtype = self.dtype
        swap = self._swap_operands
        if self._plan_device == "cpu":
            return self._cpu_runner(shapes, out_shape)
        exec_rc = self.lib.run_einsum_exec_rc
        raw_stream = _raw_stream_getter()
        get_device = torch._C._cuda_getDevice if hasattr(torch._C, "_cuda_getDevice") else torch.cuda.current_device
        f32 = torch.float32
        empty = torch.empty

        def run(*operands):
            if len(operands) != 2:
                raise ValueError("Expected exactly two operands.")
            inp0, inp1 = operands
            if inp0.shape != shapes[0] or inp1.shape != shapes[1]:
                raise ValueError(
                    f"Input shapes {inp0.shape} and {inp1.shape} do not match built shapes {self.input_shapes}.")
            if inp0.dtype != dtype or inp1.dtype != dtype:
                raise TypeError(
                    f"Input datatypes {inp0.dtype} and {inp1.dtype} do not match built datatype {dtype}.")
            dev = inp0.device
            if dev.type != 'cuda' or inp1.device != dev:
                raise ValueError(
                    f"pto_einsum: both operands must be on the same CUDA device (got {dev}, {inp1.device})")
            if not inp0.is_contiguous():
                inp0 = inp0.contiguous()
            if not inp1.is_contiguous():
                inp1 = inp1.contiguous()
            if swap:
                inp0, inp1 = inp1, inp0
            out = empty(out_shape, dtype=f32, device=dev)
            if empty_out:
                return out
            if self.lib is None:
                raise RuntimeError("pto_einsum: runner called after cleanup()")
            idx = dev.index
            wss = self._workspace
            ws = wss.get(idx) if wss else None
            if idx == get_device():
                stream = raw_stream(idx)
                if ws is None:
                    ws = self.workspace(dev, stream)
                rc = exec_rc(inp0.data_ptr(), inp1.data_ptr(), out.data_ptr(), ws, stream)
            else:
                stream = torch.cuda.current_stream(dev).cuda_stream
                if ws is None:
                    ws = self.workspace(dev, stream)
                with torch.cuda.device(dev):
                    rc = exec_rc(inp0.data_ptr(), inp1.data_ptr(), out.data_ptr(), ws, stream)
            if rc:
                self._check("run_einsum_exec")
            return out

        empty_out = prod(out_shape) == 0
        return run

    def _cpu_runner(self, shapes, out_shape):
        """Runner of a device="cpu" build: host tensors in, a host fp32 tensor out,
        computed synchronously (reference builder.py:856-875)."""
        dtype, swap = self.dtype, self._swap_operands

        def run(*operands):
            if len(operands) != 2:
                raise ValueError("Expected exactly two operands.")
            inp0, inp1 = operands
            if inp0.shape != shapes[0] or inp1.shape != shapes[1]:
                raise ValueError(
                    f"Input shapes {inp0.shape} and {inp1.shape} do not match built shapes {self.input_shapes}.")
            if inp0.dtype != dtype or inp1.dtype != dtype:
                raise TypeError(
                    f"Input datatypes {inp0.dtype} and {inp1.dtype} do not match built datatype {dtype}.")
            if inp0.device.type != 'cpu' or inp1.device.type != 'cpu':
                raise ValueError(f"pto_einsum: a device='cpu' build takes host tensors (got {inp0.device}, "
                                 f"{inp1.device})")
            if self.lib is None:
                raise RuntimeError("pto_einsum: runner called after cleanup()")
            inp0, inp1 = inp0.contiguous(), inp1.contiguous()
            if swap:
                inp0, inp1 = inp1, inp0
            # every element is written by run_einsum (no zero fill: a parallel torch
            # fill would leave its worker threads spinning against ours)
            out = torch.empty(out_shape, dtype=torch.float32, device="cpu")
            if out.numel() == 0:
                return out
            self.lib.run_einsum(inp0.data_ptr(), inp1.data_ptr(), out.data_ptr(), None)
            if self.lib.run_einsum_last_error():
                raise MemoryError(f"pto_einsum: host buffers for '{self.equation}' could not be allocated")
            return out

        return run

    def _free_workspaces(self):
        if self._workspace and self.lib is not None:
            for ws in self._workspace.values():
                self.lib.run_einsum_teardown(ctypes.c_void_p(ws))
        self._workspace = None

    def __del__(self):
        try:
            self._free_workspaces()
        except Exception:
            pass

    def cleanup(self):
        if self._composite is not None:
            for _, sub, _ in self._composite[0]:
                sub.cleanup()
            self._composite[1].cleanup()
        self._free_workspaces()
        self.lib = None
        if self.target_dir and os.path.exists(self.target_dir):
            shutil.rmtree(self.target_dir, ignore_errors=True)  # another process may share the cache


def einsum(equation: str, *operands, device="cuda", extended: bool = False):
    """One-shot two-operand einsum on CUDA; returns an fp32 tensor (builder.py:887-902).
    ``extended`` as in EinsumBuilder."""
    if len(operands) != 2:
        raise ValueError("Only exactly two operands are supported.")
    inp0, inp1 = operands
    if inp0.dtype != inp1.dtype:
        raise ValueError("Operands must have the same datatype.")
    runner = EinsumBuilder(equation, [inp0.shape, inp1.shape], inp0.dtype, device=device,
                           extended=extended).build()
    return runner(inp0, inp1)
