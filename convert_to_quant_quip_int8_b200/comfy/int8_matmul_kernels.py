"""``mm_8bit`` on the sm_100a int8 tensor-core GEMM.

Mirrors comfy/int8_matmul_kernels.py:82-110 of the reference: ``c = a @ b``
with ``a [M, K]`` int8 contiguous, ``b [K, N]`` int8 (any strides), exact
int32 result.  The kernel consumes B as ``[N, K]`` K-major, which is what
``w.t()`` of a checkpoint weight already is, so the transpose view the
reference materializes per call (comfy/quant_ops.py:471) costs nothing here.
"""

import torch

from .. import _lib as L
from .. import ops


def mm_8bit(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    assert a.shape[1] == b.shape[0], "Incompatible dimensions"
    assert a.is_contiguous(), "Matrix A must be contiguous"
    assert a.dtype == b.dtype, "Incompatible dtypes"
    assert a.dtype in [torch.int8, torch.float8_e4m3fn]
    if a.dtype != torch.int8:
        raise NotImplementedError("float8_e4m3fn mm_8bit is outside the int8 W8A8 path")
    b_nk = b.t()
    if not b_nk.is_contiguous():
        b_nk = b_nk.contiguous()
    return ops.gemm_i8(a, b_nk, out_dtype=torch.int32, act=L.QI8_ACT_NONE)
