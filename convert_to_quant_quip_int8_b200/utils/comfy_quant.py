"""``.comfy_quant`` metadata and the QuIP tensor-naming contract.

Mirrors utils/comfy_quant.py:24-48 and utils/tensor_utils.py:11-45 of the
reference and the per-layer keys written by quantization.py:651-727: a
``.comfy_quant`` uint8 tensor holding JSON (``format``, ``group_size`` for
block formats), ``weight`` int8, ``weight_scale`` fp32 (1-element scales
saved 0-d), and for transformed-space QuIP ``hadamard_quip`` int8 scalar,
``hadamard_size_out/in`` int32 scalars, ``sign_row`` / ``sign_col`` fp32.
Host-side format logic only (no kernels).
"""

import json
from typing import Dict, Optional, Tuple

import torch

BLOCK_BASED_FORMATS = ("int8_blockwise",)


def dict_to_tensor(data_dict: dict) -> torch.Tensor:
    return torch.tensor(list(json.dumps(data_dict).encode("utf-8")), dtype=torch.uint8)


def tensor_to_dict(tensor: torch.Tensor) -> dict:
    if tensor.dtype != torch.uint8:
        raise ValueError(f"Expected uint8 tensor, got {tensor.dtype}")
    return json.loads(bytes(tensor.tolist()).decode("utf-8"))


def create_comfy_quant_tensor(format_type: str, block_size: Optional[int] = None,
                              full_precision_matrix_mult: Optional[bool] = None) -> torch.Tensor:
    cfg = {"format": format_type}
    if block_size is not None and format_type in BLOCK_BASED_FORMATS:
        cfg["group_size"] = block_size
    if full_precision_matrix_mult is True:
        cfg["full_precision_matrix_mult"] = True
    return dict_to_tensor(cfg)


def normalize_tensorwise_scales(tensors: Dict[str, torch.Tensor], enabled: bool = True
                                ) -> Tuple[Dict[str, torch.Tensor], int]:
    """1-element scale tensors become 0-d scalars; everything is made contiguous."""
    out, count = {}, 0
    suffixes = (".weight_scale", ".input_scale", ".scale_weight", ".scale_input")
    for key, t in tensors.items():
        if enabled and key.endswith(suffixes) and t.numel() == 1 and t.ndim > 0:
            out[key] = torch.tensor(t.item(), dtype=t.dtype)
            count += 1
            continue
        out[key] = t if t.is_contiguous() else t.contiguous()
    return out, count


def quip_layer_tensors(base_name: str, result: tuple, block_size: int = 128) -> Dict[str, torch.Tensor]:
    """Checkpoint tensors of one converted layer, from a ``QuIPInt8Converter.convert``
    result tuple, with the names and dtypes of quantization.py:651-727."""
    q, scale, _deq, smooth, s_u, s_v, hadamard_quip, size_out, size_in = result
    t = {f"{base_name}.weight": q.to("cpu")}
    if smooth is not None:
        t[f"{base_name}.smooth_factors"] = smooth.to("cpu", torch.float32)
    if hadamard_quip and s_u is not None and s_v is not None:
        t[f"{base_name}.hadamard_quip"] = torch.tensor(1, dtype=torch.int8)
        t[f"{base_name}.hadamard_size_out"] = torch.tensor(size_out, dtype=torch.int32)
        t[f"{base_name}.hadamard_size_in"] = torch.tensor(size_in, dtype=torch.int32)
        t[f"{base_name}.sign_row"] = s_u.to("cpu", torch.float32)
        t[f"{base_name}.sign_col"] = s_v.to("cpu", torch.float32)
    fmt = "int8_blockwise" if scale.dim() >= 3 else "int8_tensorwise"
    t[f"{base_name}.weight_scale"] = scale.to("cpu", torch.float32).detach().clone()
    t[f"{base_name}.comfy_quant"] = create_comfy_quant_tensor(fmt, block_size if fmt in BLOCK_BASED_FORMATS else None)
    return t
