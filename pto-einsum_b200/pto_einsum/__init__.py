"""pto_einsum: a two-operand einsum for NVIDIA B200 (sm_100a).

Drop-in for the pto-einsum API (src/pto_einsum/__init__.py:12-15):

    einsum(equation, a, b, device="cuda")      -> fp32 result tensor
    EinsumBuilder(equation, shapes, dtype)     -> .build() returns a reusable runner

The equation parser and transpose -> batched matmul -> transpose planner keep
the reference's behaviour (plan-identical recipes). Execution is hand-written
sm_100a CUDA (TMA + tcgen05/TMEM GEMM, 128-bit streaming kernels) behind a
per-equation C ABI cached on disk.

Example:
    >>> from pto_einsum import einsum
    >>> c = einsum("ij, jk -> ik", a, b)            # a, b are CUDA tensors
"""

from ._core import INCLUDE_DIR
from .builder import EinsumBuilder, einsum

__all__ = ["einsum", "EinsumBuilder", "INCLUDE_DIR"]
__version__ = "0.1.0"
