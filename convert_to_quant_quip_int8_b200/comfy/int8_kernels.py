"""INT8 kernel wrappers with the signatures of comfy/int8_kernels.py.

Each function keeps the reference's argument meaning, shape asserts and
return dtypes; the arithmetic runs in libqi8 (see include/qi8.h):

* ``act_quant`` / ``weight_quant``       Triton act_quant / weight_quant
                                           (comfy/int8_kernels.py:72-253)
* ``act_dequant`` / ``weight_dequant``   (:126-179, :256-330)
* ``int8_gemm`` / ``int8_addmm``         block-K promoted GEMM (:335-647)
* ``int8_gemm_quant`` / ``int8_addmm_quant``  GEMM with the output
                                           requantized in the epilogue (:684-1089)
* ``int8_gelu``                          fused int8 GELU (:1122-1312)
* ``quip_int8_matmul``                   transformed-space QuIP linear
                                           (:1374-1452), as W8A8: K1 rotate +
                                           per-token quant, tcgen05 GEMM, K3
"""

from typing import Optional, Tuple

import torch

from .. import _lib as L
from .. import ops


def act_quant(x: torch.Tensor, block_size: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    assert x.is_contiguous(), "Input tensor must be contiguous"
    assert x.size(-1) % block_size == 0, \
        f"Last dimension size must be divisible by block_size (block_size={block_size})"
    return ops.quant_rows(x, L.QI8_Q_BLOCK, block_size)


def act_dequant(x: torch.Tensor, s: torch.Tensor, block_size: int = 128,
                output_dtype: torch.dtype = None) -> torch.Tensor:
    assert x.is_contiguous() and s.is_contiguous(), "Input tensors must be contiguous"
    assert x.size(-1) % block_size == 0, \
        f"Last dimension size must be divisible by block_size (block_size={block_size})"
    if output_dtype is None:
        output_dtype = torch.get_default_dtype()
    return ops.dequant(x, s, L.QI8_S_ROW_KBLOCK, block_size, output_dtype)


def weight_quant(x: torch.Tensor, block_size: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    assert x.is_contiguous(), "Input tensor must be contiguous"
    assert x.dim() == 2, "Input tensor must have 2 dimensions"
    M, N = x.size()
    assert M % block_size == 0 and N % block_size == 0, \
        f"Dimensions must be divisible by block_size={block_size}, got shape {x.shape}"
    if block_size != 128:
        raise NotImplementedError("weight_quant supports block_size=128")
    return ops.quant_weight(x, L.QI8_S_TILE128)


def weight_dequant(x: torch.Tensor, s: torch.Tensor, block_size: int = 128,
                   output_dtype: torch.dtype = None) -> torch.Tensor:
    assert x.is_contiguous() and s.is_contiguous(), "Input tensors must be contiguous"
    assert x.dim() == 2 and s.dim() == 2, "Input tensors must have 2 dimensions"
    if output_dtype is None:
        output_dtype = torch.get_default_dtype()
    return ops.dequant(x, s, L.QI8_S_TILE128, block_size, output_dtype)


def _block_gemm(a, a_s, b, b_s, bias, input_block_size, out_dtype):
    assert a.is_contiguous() and b.is_contiguous(), "Input tensors must be contiguous"
    assert a_s.is_contiguous() and b_s.is_contiguous(), "Scaling factor tensors must be contiguous"
    assert b.dim() == 2, f"Expected b to be 2D, got shape {b.shape}"
    K = a.size(-1)
    N = b.shape[0]
    assert b.size(1) == K, f"Shape mismatch: b.shape={b.shape}, expected [..., {K}]"
    assert input_block_size == 128, "block size must be 128"
    M = a.numel() // K
    a_kind = L.QI8_S_ROW_KBLOCK if a_s.numel() == M * (K // 128) else ops.scale_kind(a_s, M, K, False)
    b_kind = ops.scale_kind(b_s, N, K, True)
    if bias is not None:
        assert bias.is_contiguous(), "Bias tensor must be contiguous"
        assert bias.dim() == 1 and bias.size(0) == N, f"Bias must be 1D with length {N}, got shape {bias.shape}"
    return ops.gemm_i8(a, b, a_s, a_kind, b_s, b_kind, bias, out_dtype)


def int8_gemm(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor,
              input_block_size: int = 128, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """``C = A B^T`` with per-128-block scales; fp16 output like the reference."""
    return _block_gemm(a, a_s, b, b_s, None, input_block_size, out_dtype)


def int8_addmm(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor,
               bias: Optional[torch.Tensor] = None, input_block_size: int = 128,
               out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """``C = A B^T + bias`` with per-128-block scales; fp16 output like the reference."""
    return _block_gemm(a, a_s, b, b_s, bias, input_block_size, out_dtype)


def _quant_gemm(a, a_s, b, b_s, bias, out_block_size, input_block_size):
    assert a.is_contiguous() and b.is_contiguous(), "Input tensors must be contiguous"
    assert a_s.is_contiguous() and b_s.is_contiguous(), "Scaling tensors must be contiguous"
    assert b.dim() == 2, f"Expected b to be 2D, got shape {b.shape}"
    K = a.size(-1)
    N = b.shape[0]
    assert b.size(1) == K, f"Shape mismatch: b.shape={b.shape}, expected [..., {K}]"
    assert N % out_block_size == 0, f"N={N} must be divisible by out_block_size={out_block_size}"
    if out_block_size != 128 or input_block_size != 128:
        raise NotImplementedError("the fused requantizing GEMM uses 128-element blocks")
    return ops.gemm_i8_quant(a, b, a_s, b_s, bias, out_block_size)


def int8_gemm_quant(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor,
                    out_block_size: int = 128, input_block_size: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """``C_int8, C_scale = quantize(A @ B)`` in one kernel: the block-promoted
    GEMM's epilogue requantizes every (row, 128-column block) of the fp32
    result (comfy/int8_kernels.py:920-996)."""
    return _quant_gemm(a, a_s, b, b_s, None, out_block_size, input_block_size)


def int8_addmm_quant(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor,
                     bias: Optional[torch.Tensor] = None, out_block_size: int = 128,
                     input_block_size: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """``C_int8, C_scale = quantize(A @ B + bias)`` in one kernel (:998-1089)."""
    if bias is not None:
        assert bias.is_contiguous(), "Bias tensor must be contiguous"
    return _quant_gemm(a, a_s, b, b_s, bias, out_block_size, input_block_size)


def int8_gelu(x: torch.Tensor, s_x: torch.Tensor, block_size: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """``y_int8, y_scale = quantize(gelu(dequantize(x, s_x)))`` in one kernel (:1234-1312)."""
    assert x.is_contiguous(), "Input tensor must be contiguous"
    assert s_x.is_contiguous(), "Scale tensor must be contiguous"
    assert x.size(-1) % block_size == 0, f"Last dimension must be divisible by block_size={block_size}"
    if block_size != 128:
        raise NotImplementedError("the fused int8 GELU uses 128-element blocks")
    return ops.int8_gelu(x, s_x, block_size)


def quip_int8_matmul(x: torch.Tensor, Q: torch.Tensor, scale: torch.Tensor, s_u: torch.Tensor,
                     s_v: torch.Tensor, block_size: int = 128) -> torch.Tensor:
    """Transformed-space QuIP linear ``y = FWHT(FWHT(x * s_v) @ (scale * Q)^T) * s_u``.

    The reference (comfy/int8_kernels.py:1374-1452) multiplies fp32 rotated
    activations by the dequantized weight; this W8A8 version quantizes the
    rotated activations per token (K1), runs the int8 tensor-core GEMM with
    the ``x_s * w_s`` epilogue (K2) and un-rotates the fp32 result (K3).
    Returns fp32 ``[M, N]`` like the reference.
    """
    M, K = x.shape
    N = Q.shape[0]
    scale = scale.to(device=x.device, dtype=torch.float32).contiguous()
    if scale.dim() > 1:
        scale = scale.squeeze()
    if scale.numel() == 1:
        scale = scale.reshape(()).expand(N).contiguous()
    xq, xs = ops.rotate_quant_rows(x.contiguous(), s_v, K)
    y_had = ops.gemm_i8(xq, Q.contiguous().to(torch.int8), xs, L.QI8_S_ROW, scale, L.QI8_S_ROW, None,
                        torch.float32)
    return ops.unrotate_rows(y_had, s_u, N, None, torch.float32)
