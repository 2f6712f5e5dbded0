"""Hadamard helpers (mirror of utils/hadamard.py in the reference).

``fast_hadamard_transform`` and friends run the sm_100a kernels in fp32;
the reference's optional bf16 "mixed" core (utils/hadamard.py:190-253) is a
lossy GPU-only path and is not reproduced: ``use_mixed_precision`` is
accepted and ignored.
"""

import math
from typing import Optional

import torch

from .. import ops
from ..comfy import hadamard_kernels as _hk


def is_power_of_two(n: int) -> bool:
    return (n > 0) and (n & (n - 1) == 0)


def next_power_of_two(n: int) -> int:
    if n <= 0:
        return 1
    return 2 ** (n - 1).bit_length()


def hadamard_matrix(n: int) -> torch.Tensor:
    """Normalized Sylvester Hadamard matrix (utils/hadamard.py:309-336), built on the host."""
    if not is_power_of_two(n):
        raise ValueError(f"n must be a power of 2, got {n}")
    h = torch.ones((1, 1))
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0) / math.sqrt(2)
    return h


def fast_hadamard_transform(x: torch.Tensor, normalize: bool = True, inplace: bool = False,
                            use_mixed_precision: Optional[bool] = None) -> torch.Tensor:
    n = x.shape[-1]
    if not is_power_of_two(n):
        raise ValueError(f"Last dimension must be a power of 2, got {n}")
    y = ops.fwht_rows(x, n, normalize=normalize).reshape(x.shape)
    if inplace and x.dtype == torch.float32:
        x.copy_(y)
        return x
    return y


def fast_hadamard_transform_with_signs(x: torch.Tensor, sign_row: Optional[torch.Tensor] = None,
                                       sign_col: Optional[torch.Tensor] = None,
                                       normalize: bool = True) -> torch.Tensor:
    """1-D FWHT of ``x * sign_row[:, None] * sign_col[None, :]`` (utils/hadamard.py:411-464)."""
    return _hk.triton_hadamard_transform_with_signs(x, sign_row, sign_col, normalize)


def fast_hadamard_transform_2d(x: torch.Tensor, normalize: bool = True, inplace: bool = False) -> torch.Tensor:
    return _hk.fast_hadamard_transform_2d(x, normalize, inplace)


def fast_hadamard_transform_2d_with_signs(x, sign_row=None, sign_col=None, normalize: bool = True):
    return _hk.fast_hadamard_transform_2d_with_signs(x, sign_row, sign_col, normalize)
