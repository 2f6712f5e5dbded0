"""Fast Walsh-Hadamard transforms (mirror of comfy/hadamard_kernels.py).

The reference runs one HBM ping-pong Triton launch per butterfly stage plus a
normalize pass (comfy/hadamard_kernels.py:244-373); here each row is
transformed in one pass on-chip (``qi8_fwht_rows``), and the row-dimension
half of the 2-D transform uses the column kernel (``qi8_fwht_cols``).
Results equal the reference's fp32 CPU core bit for bit.
"""

import math
from typing import Optional

import torch

from .. import ops

HAS_TRITON_HADAMARD = False  # API compatibility: the transforms below are libqi8 kernels


def _is_pow2(n: int) -> bool:
    return n > 0 and (n & (n - 1)) == 0


def _rows_fp32(x: torch.Tensor) -> torch.Tensor:
    return x if x.dtype == torch.float32 else x.float()


def triton_hadamard_transform(x: torch.Tensor, normalize: bool = True,
                              output: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FWHT over the last dimension (name kept from the reference)."""
    n = x.shape[-1]
    if not _is_pow2(n):
        raise ValueError(f"Last dimension must be a power of 2, got {n}")
    y = ops.fwht_rows(x, n, normalize=normalize)
    if output is not None:
        output.copy_(y.reshape(output.shape))
        return output
    return y.reshape(x.shape)


def fast_hadamard_transform(x: torch.Tensor, normalize: bool = True) -> torch.Tensor:
    return triton_hadamard_transform(x, normalize=normalize)


def triton_hadamard_transform_with_signs(x: torch.Tensor, sign_row: Optional[torch.Tensor] = None,
                                         sign_col: Optional[torch.Tensor] = None, normalize: bool = True,
                                         output: Optional[torch.Tensor] = None) -> torch.Tensor:
    """1-D FWHT of ``x * sign_row[:, None] * sign_col[None, :]`` (signs before the transform)."""
    n = x.shape[-1]
    if not _is_pow2(n):
        raise ValueError(f"Last dimension must be a power of 2, got {n}")
    xs = x
    if sign_row is not None:
        xs = _rows_fp32(xs) * sign_row.to(xs.device, torch.float32).unsqueeze(-1)
    y = ops.fwht_rows(xs, n, pre_sign=sign_col, normalize=normalize).reshape(x.shape)
    if output is not None:
        output.copy_(y)
        return output
    return y


def fast_hadamard_transform_with_signs(x: torch.Tensor, sign_row: Optional[torch.Tensor] = None,
                                       sign_col: Optional[torch.Tensor] = None,
                                       normalize: bool = True) -> torch.Tensor:
    """2-D transform when both trailing dims are powers of two >= 64 and the
    signs match them (comfy/hadamard_kernels.py:499-538), else 1-D."""
    if x.dim() >= 2:
        r, c = x.shape[-2], x.shape[-1]
        if r >= 64 and c >= 64 and _is_pow2(r) and _is_pow2(c):
            if (sign_row is None or sign_row.shape[-1] == r) and (sign_col is None or sign_col.shape[-1] == c):
                return fast_hadamard_transform_2d_with_signs(x, sign_row, sign_col, normalize)
    return triton_hadamard_transform_with_signs(x, sign_row, sign_col, normalize)


def fast_hadamard_transform_2d(x: torch.Tensor, normalize: bool = True, inplace: bool = False) -> torch.Tensor:
    """``H X H^T``: last-dim FWHT, then row-dim FWHT, un-normalized, then one
    fp32 division by ``sqrt(rows * cols)`` (comfy/hadamard_kernels.py:541-575)."""
    r, c = x.shape[-2], x.shape[-1]
    if not _is_pow2(r):
        raise ValueError(f"Second-to-last dimension must be power of 2, got {r}")
    if not _is_pow2(c):
        raise ValueError(f"Last dimension must be power of 2, got {c}")
    y = ops.fwht_rows(x, c, normalize=False).reshape(-1, r, c)
    for b in range(y.shape[0]):
        ops.fwht_cols_(y[b], 2 if normalize else 0, math.sqrt(r * c))
    y = y.reshape(x.shape)
    if inplace and x.dtype == torch.float32:
        x.copy_(y)
        return x
    return y


def fast_hadamard_transform_2d_with_signs(x: torch.Tensor, sign_row: Optional[torch.Tensor] = None,
                                          sign_col: Optional[torch.Tensor] = None,
                                          normalize: bool = True) -> torch.Tensor:
    """``H (D1 X D2) H^T`` (signs first, then the 2-D transform)."""
    xs = _rows_fp32(x)
    if sign_row is not None:
        xs = xs * sign_row.to(xs.device, torch.float32).unsqueeze(-1)
    if sign_col is not None:
        xs = xs * sign_col.to(xs.device, torch.float32).unsqueeze(-2)
    return fast_hadamard_transform_2d(xs.contiguous(), normalize=normalize)


def inverse_hadamard_transform_with_signs(x: torch.Tensor, sign_row: Optional[torch.Tensor] = None,
                                          sign_col: Optional[torch.Tensor] = None,
                                          orig_shape: Optional[tuple] = None,
                                          normalize: bool = True) -> torch.Tensor:
    """1-D FWHT, then the signs, then slicing (comfy/hadamard_kernels.py:607-639)."""
    y = ops.fwht_rows(x, x.shape[-1], post_sign=sign_col, normalize=normalize).reshape(x.shape)
    if sign_row is not None:
        y = y * sign_row.to(y.device, torch.float32).unsqueeze(-1)
    if orig_shape is not None:
        y = y[tuple(slice(0, s) for s in orig_shape)]
    return y


def inverse_hadamard_transform_2d_with_signs(x: torch.Tensor, sign_row: Optional[torch.Tensor] = None,
                                             sign_col: Optional[torch.Tensor] = None,
                                             orig_rows: Optional[int] = None, orig_cols: Optional[int] = None,
                                             normalize: bool = True) -> torch.Tensor:
    """2-D transform, then signs, then slicing (comfy/hadamard_kernels.py:642-693)."""
    y = fast_hadamard_transform_2d(_rows_fp32(x).contiguous(), normalize=normalize)
    if sign_row is not None:
        y = y * sign_row.to(y.device, torch.float32).view(*([1] * (y.dim() - 2)), -1, 1)
    if sign_col is not None:
        y = y * sign_col.to(y.device, torch.float32).view(*([1] * (y.dim() - 2)), 1, -1)
    sl = [slice(None)] * y.dim()
    if orig_rows is not None:
        sl[-2] = slice(0, orig_rows)
    if orig_cols is not None:
        sl[-1] = slice(0, orig_cols)
    return y[tuple(sl)]


__all__ = ["HAS_TRITON_HADAMARD", "triton_hadamard_transform", "fast_hadamard_transform",
           "fast_hadamard_transform_with_signs", "fast_hadamard_transform_2d",
           "fast_hadamard_transform_2d_with_signs", "inverse_hadamard_transform_with_signs",
           "inverse_hadamard_transform_2d_with_signs"]
