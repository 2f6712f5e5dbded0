"""Axis-wise / tensor-wise INT8 quantization (utils/float_utils.py of the reference).

Same signatures and results (bit-exact): ``scale = (amax/127).clamp(min=1e-30)``
in fp32, ``q = round_half_even(x * (1/scale)).clamp(-128, 127)``; computed
in one pass by libqi8 (``qi8_quant_rows`` / ``qi8_quant_weight``).
"""

from typing import Optional

import torch

from .. import _lib as L
from .. import ops


def _no_percentile(p):
    if p is not None and 0.5 < p < 1.0:
        raise NotImplementedError("percentile scaling (outlier_percentile < 1) is not part of the W8A8 path")


def quantize_int8_axiswise(x: torch.Tensor, dim: int = -1,
                           outlier_percentile: Optional[float] = None) -> tuple:
    """Per-row absmax int8 quantization along ``dim``; returns ``(q, scale)``
    with ``scale`` keeping a size-1 ``dim`` like the reference."""
    _no_percentile(outlier_percentile)
    if dim not in (-1, x.dim() - 1):
        xt = x.transpose(dim, -1)
        q, s = ops.quant_rows(xt.contiguous(), L.QI8_Q_TOKEN)
        return q.transpose(dim, -1), s.transpose(dim, -1)
    return ops.quant_rows(x, L.QI8_Q_TOKEN)


def quantize_int8_tensorwise(x: torch.Tensor, outlier_percentile: Optional[float] = None) -> tuple:
    """Whole-tensor absmax int8 quantization; returns ``(q, scale)`` with a 0-d scale."""
    _no_percentile(outlier_percentile)
    q, s = ops.quant_weight(x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x, L.QI8_S_SCALAR)
    return q.reshape(x.shape), s
