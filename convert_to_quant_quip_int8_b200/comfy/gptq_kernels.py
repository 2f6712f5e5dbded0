"""GPTQ block kernel with the interface of comfy/gptq_kernels.py.

``triton_gptq_quant_block(W, Hinv, scale) -> (Q, Err)`` keeps the
reference's name, argument meaning and return dtypes (comfy/gptq_kernels.py:
87-124): ``W`` [M, block] fp32 is updated in place (as the reference does,
a non-contiguous ``W`` is first copied, so the caller's view is then left
unchanged), ``Hinv`` [block, block] is the block of the inverse Hessian's
Cholesky factor, ``scale`` a scalar or [M, 1].  The arithmetic runs in
``qi8_gptq_quant_block`` on the GPU.
"""

from typing import Tuple

import torch

from .. import _lib as L

HAS_TRITON = True  # the reference's flag: this module's kernel is always available


def triton_gptq_quant_block(W: torch.Tensor, Hinv: torch.Tensor, scale) -> Tuple[torch.Tensor, torch.Tensor]:
    L.require_cuda(W, Hinv)
    M, B = W.shape
    Q = torch.empty((M, B), device=W.device, dtype=torch.int8)
    Err = torch.empty((M, B), device=W.device, dtype=torch.float32)
    if not W.is_contiguous():
        W = W.contiguous()
    assert W.dtype == torch.float32, "W must be fp32"
    Hinv = Hinv.to(torch.float32)
    if Hinv.stride(1) != 1:
        Hinv = Hinv.contiguous()
    if not isinstance(scale, torch.Tensor):
        scale = torch.tensor([float(scale)], device=W.device)
    scalar = scale.numel() == 1
    sc = scale.to(device=W.device, dtype=torch.float32).reshape(-1).contiguous()
    L.check(L.load().qi8_gptq_quant_block(L.ptr(W), M, B, W.stride(0), L.ptr(Hinv), Hinv.stride(0), L.ptr(sc),
                                          int(scalar), L.ptr(Q), B, L.ptr(Err), B, L.stream_ptr(W.device)),
            "qi8_gptq_quant_block")
    return Q, Err
