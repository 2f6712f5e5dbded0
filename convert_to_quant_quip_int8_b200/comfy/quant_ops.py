"""``QuantizedTensor`` and INT8 layouts -- the ComfyUI operator surface.

Mirrors comfy/quant_ops.py of the reference (``QuantizedTensor`` :94-175,
``BlockWiseINT8Layout`` :260-317, ``TensorWiseINT8Layout`` :319-328,
``AxisWiseINT8Layout`` :330-339, ``QUANT_ALGOS`` / ``LAYOUTS`` :341-356 and the
``aten`` handlers :373-475): same names, layout parameters, registry and
dispatch order.  Differences, all on the hot path:

* every quantize / dequantize / GEMM runs in libqi8 on sm_100a; a CPU tensor
  raises instead of falling back;
* ``optimized_linear`` accepts the QuIP per-row ``[N, 1]`` tensorwise scale
  (the reference's broadcast ``x_s * w_s.unsqueeze(0)`` fails for it unless
  T == N) and never materializes ``w_q.t().contiguous()``;
* a ``BlockWiseINT8Layout`` weight carrying the QuIP block-requant scale
  ``[N, K/128(, 1)]`` runs W8A8 (per-token activations, per-128-K-block
  promotion) for plain inputs -- the reference has no consumer for that
  layout;
* ``QuIPHadamardINT8Layout`` (new) consumes transformed-space checkpoints
  (``sign_row`` / ``sign_col`` / ``hadamard_size_*``) as a W8A8 linear;
* ``F.linear`` reaches the linear handlers through ``__torch_function__``
  (in the reference it decomposes into ``t`` + ``mm`` before dispatch).
"""

from __future__ import annotations

import logging
from typing import Dict, Tuple

import torch

from .. import _lib as L
from .. import ops

_LAYOUT_REGISTRY: Dict = {}
_GENERIC_UTILS: Dict = {}

_HAS_TRITON_INT8 = False  # kept for API compatibility: no Triton in this package
_HAS_QI8 = True


def register_layout_op(torch_op, layout_type):
    def decorator(handler_func):
        _LAYOUT_REGISTRY.setdefault(torch_op, {})[layout_type] = handler_func
        return handler_func
    return decorator


def register_generic_util(torch_op):
    def decorator(handler_func):
        _GENERIC_UTILS[torch_op] = handler_func
        return handler_func
    return decorator


def _get_layout_from_args(args):
    for arg in args:
        if isinstance(arg, QuantizedTensor):
            return arg._layout_type
        if isinstance(arg, (list, tuple)):
            for item in arg:
                if isinstance(item, QuantizedTensor):
                    return item._layout_type
    return None


def _map_tensors(params, fn):
    return {k: (fn(v) if isinstance(v, torch.Tensor) else v) for k, v in params.items()}


class QuantizedLayout:
    @classmethod
    def quantize(cls, tensor, **kwargs) -> Tuple[torch.Tensor, Dict]:
        raise NotImplementedError(f"{cls.__name__} must implement quantize()")

    @staticmethod
    def dequantize(qdata, **layout_params) -> torch.Tensor:
        raise NotImplementedError("TensorLayout must implement dequantize()")

    @classmethod
    def get_plain_tensors(cls, qtensor):
        raise NotImplementedError(f"{cls.__name__} must implement get_plain_tensors()")


class QuantizedTensor(torch.Tensor):
    """Wrapper subclass holding int8 ``_qdata`` plus layout parameters."""

    @staticmethod
    def __new__(cls, qdata, layout_type, layout_params):
        return torch.Tensor._make_wrapper_subclass(cls, qdata.shape, device=qdata.device,
                                                   dtype=qdata.dtype, requires_grad=False)

    def __init__(self, qdata, layout_type, layout_params):
        self._qdata = qdata
        self._layout_type = layout_type
        self._layout_params = layout_params

    def __repr__(self):
        return f"QuantizedTensor(shape={self.shape}, layout={self._layout_type})"

    @property
    def layout_type(self):
        return self._layout_type

    def __tensor_flatten__(self):
        tensor_keys = [k for k, v in self._layout_params.items() if isinstance(v, torch.Tensor)]
        ctx = {"layout_type": self._layout_type, "tensor_param_keys": tensor_keys,
               "non_tensor_params": {k: v for k, v in self._layout_params.items()
                                     if not isinstance(v, torch.Tensor)}}
        inner = ["_qdata"]
        for k in tensor_keys:
            object.__setattr__(self, f"_layout_param_{k}", self._layout_params[k])
            inner.append(f"_layout_param_{k}")
        return inner, ctx

    @staticmethod
    def __tensor_unflatten__(inner_tensors, ctx, outer_size, outer_stride):
        params = dict(ctx["non_tensor_params"])
        for k in ctx["tensor_param_keys"]:
            params[k] = inner_tensors[f"_layout_param_{k}"]
        return QuantizedTensor(inner_tensors["_qdata"], ctx["layout_type"], params)

    @classmethod
    def from_float(cls, tensor, layout_type, **quantize_kwargs) -> "QuantizedTensor":
        qdata, params = LAYOUTS[layout_type].quantize(tensor, **quantize_kwargs)
        return cls(qdata, layout_type, params)

    def dequantize(self) -> torch.Tensor:
        return LAYOUTS[self._layout_type].dequantize(self._qdata, **self._layout_params)

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        # aten.linear is CompositeImplicitAutograd: below the Python
        # function layer it decomposes into t + mm before __torch_dispatch__
        # sees it, so F.linear is routed to the registered linear handlers here.
        kwargs = kwargs or {}
        if func is torch.nn.functional.linear:
            layout = _get_layout_from_args(args)
            handler = _LAYOUT_REGISTRY.get(torch.ops.aten.linear.default, {}).get(layout)
            if handler is not None:
                return handler(torch.ops.aten.linear.default, args, kwargs)
        return torch._C._disabled_torch_function_impl(func, types, args, kwargs)

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func in _GENERIC_UTILS:
            return _GENERIC_UTILS[func](func, args, kwargs)
        layout_type = _get_layout_from_args(args)
        if layout_type and func in _LAYOUT_REGISTRY:
            handler = _LAYOUT_REGISTRY[func].get(layout_type)
            if handler:
                return handler(func, args, kwargs)
        return cls._dequant_and_fallback(func, args, kwargs)

    @classmethod
    def _dequant_and_fallback(cls, func, args, kwargs):
        def deq(a):
            if isinstance(a, QuantizedTensor):
                return a.dequantize()
            if isinstance(a, (list, tuple)):
                return type(a)(deq(x) for x in a)
            return a
        return func(*deq(args), **deq(kwargs))

    def data_ptr(self):
        return self._qdata.data_ptr()

    def is_pinned(self):
        return self._qdata.is_pinned()

    def is_contiguous(self, *args, **kwargs):
        return self._qdata.is_contiguous(*args, **kwargs)

    def storage(self):
        return self._qdata.storage()


def _new_like(qt, qdata, params=None):
    return QuantizedTensor(qdata, qt._layout_type, params if params is not None else
                           _map_tensors(qt._layout_params, lambda v: v.clone()))


def _device_transfer(qt, target_device, target_dtype=None):
    if target_device is not None:
        target_device = torch.device(target_device)
        if target_device != qt._qdata.device:
            params = _map_tensors(qt._layout_params, lambda v: v.to(device=target_device))
            if target_dtype is not None:
                params["orig_dtype"] = target_dtype
            return QuantizedTensor(qt._qdata.to(device=target_device), qt._layout_type, params)
    return qt


@register_generic_util(torch.ops.aten.detach.default)
def generic_detach(func, args, kwargs):
    qt = args[0]
    if isinstance(qt, QuantizedTensor):
        return _new_like(qt, qt._qdata.detach())
    return func(*args, **kwargs)


@register_generic_util(torch.ops.aten.clone.default)
def generic_clone(func, args, kwargs):
    qt = args[0]
    if isinstance(qt, QuantizedTensor):
        return _new_like(qt, qt._qdata.clone())
    return func(*args, **kwargs)


@register_generic_util(torch.ops.aten._to_copy.default)
def generic_to_copy(func, args, kwargs):
    qt = args[0]
    if isinstance(qt, QuantizedTensor):
        return _device_transfer(qt, kwargs.get("device"), kwargs.get("dtype"))
    return func(*args, **kwargs)


@register_generic_util(torch.ops.aten.to.dtype_layout)
def generic_to_dtype_layout(func, args, kwargs):
    qt = args[0]
    if isinstance(qt, QuantizedTensor):
        return _device_transfer(qt, kwargs.get("device"), kwargs.get("dtype"))
    return func(*args, **kwargs)


@register_generic_util(torch.ops.aten.to.dtype)
def generic_to_dtype(func, args, kwargs):
    src = args[0]
    if isinstance(src, QuantizedTensor):
        src._layout_params["orig_dtype"] = args[1] if len(args) > 1 else kwargs.get("dtype")
        return src
    return func(*args, **kwargs)


@register_generic_util(torch.ops.aten.copy_.default)
def generic_copy_(func, args, kwargs):
    dst, src = args[0], args[1]
    non_blocking = args[2] if len(args) > 2 else False
    if isinstance(dst, QuantizedTensor):
        if isinstance(src, QuantizedTensor):
            dst._qdata.copy_(src._qdata, non_blocking=non_blocking)
            dst._layout_type = src._layout_type
            keep = dst._layout_params["orig_dtype"]
            for k, v in src._layout_params.items():
                if isinstance(v, torch.Tensor):
                    dst._layout_params[k].copy_(v, non_blocking=non_blocking)
                else:
                    dst._layout_params[k] = v
            dst._layout_params["orig_dtype"] = keep
        else:
            dst._qdata.copy_(src)
        return dst
    return func(*args, **kwargs)


@register_generic_util(torch.ops.aten._has_compatible_shallow_copy_type.default)
def generic_has_compatible_shallow_copy_type(func, args, kwargs):
    return True


@register_generic_util(torch.ops.aten.empty_like.default)
def generic_empty_like(func, args, kwargs):
    qt = args[0]
    if isinstance(qt, QuantizedTensor):
        hp_dtype = kwargs.pop("dtype", qt._layout_params["orig_dtype"])
        qdata = torch.empty_like(qt._qdata, **kwargs)
        device = kwargs.get("device", qdata.device)
        params = _map_tensors(qt._layout_params, lambda v: v.to(device=device))
        params["orig_dtype"] = hp_dtype
        return QuantizedTensor(qdata, qt._layout_type, params)
    return func(*args, **kwargs)


# --------------------------------------------------------------- layouts
class BlockWiseINT8Layout(QuantizedLayout):
    """128x128-tile weights / per-(row, 128-block) activations (Triton semantics:
    scale = amax/127 (weights floored at 1e-8), truncating int8 conversion)."""

    @classmethod
    def quantize(cls, tensor, scale=None, block_size=128, is_weight=False, **kwargs):
        L.require_cuda(tensor)
        orig_dtype = tensor.dtype
        tensor = tensor.contiguous()
        if scale is not None:
            raise NotImplementedError("static (pre-computed) block scales are not supported")
        if is_weight:
            from .int8_kernels import weight_quant
            qdata, scale = weight_quant(tensor, block_size=block_size)
        else:
            from .int8_kernels import act_quant
            qdata, scale = act_quant(tensor, block_size=block_size)
        return qdata, {"scale": scale.to(torch.float32), "block_size": block_size, "is_weight": is_weight,
                       "orig_dtype": orig_dtype}

    @staticmethod
    def dequantize(qdata, scale, block_size, is_weight=False, orig_dtype=None, output_dtype=None, **kwargs):
        out_dtype = output_dtype if output_dtype is not None else orig_dtype
        qdata = qdata.contiguous()
        scale = scale.contiguous()
        if is_weight:
            N, K = qdata.shape
            if scale.numel() == (N // block_size) * (K // block_size):
                return ops.dequant(qdata, scale, L.QI8_S_TILE128, block_size, out_dtype)
            # QuIP block requant scale [N, K/bs(, 1)]: per row x K block
            return ops.dequant(qdata, scale, L.QI8_S_ROW_KBLOCK, block_size, out_dtype)
        return ops.dequant(qdata, scale, L.QI8_S_ROW_KBLOCK, block_size, out_dtype)

    @classmethod
    def get_plain_tensors(cls, qtensor):
        p = qtensor._layout_params
        return qtensor._qdata, p["scale"], p["block_size"], p["is_weight"]


class TensorWiseINT8Layout(QuantizedLayout):
    @classmethod
    def quantize(cls, tensor, scale=None, **kwargs):
        from ..utils.float_utils import quantize_int8_tensorwise
        qdata, scale = quantize_int8_tensorwise(tensor)
        return qdata, {"scale": scale, "orig_dtype": tensor.dtype}

    @staticmethod
    def dequantize(qdata, scale, orig_dtype, **kwargs):
        kind = L.QI8_S_SCALAR if scale.numel() == 1 else L.QI8_S_ROW
        return ops.dequant(qdata, scale, kind, 0, orig_dtype)

    @classmethod
    def get_plain_tensors(cls, qtensor):
        return qtensor._qdata, qtensor._layout_params["scale"]


class AxisWiseINT8Layout(QuantizedLayout):
    @classmethod
    def quantize(cls, tensor, scale=None, **kwargs):
        from ..utils.float_utils import quantize_int8_axiswise
        qdata, scale = quantize_int8_axiswise(tensor)
        return qdata, {"scale": scale.squeeze(1), "orig_dtype": tensor.dtype}

    @staticmethod
    def dequantize(qdata, scale, orig_dtype, **kwargs):
        # the reference multiplies by a 2-D fp32 scale, which promotes to fp32
        return ops.dequant(qdata, scale, L.QI8_S_ROW, 0, torch.float32)

    @classmethod
    def get_plain_tensors(cls, qtensor):
        return qtensor._qdata, qtensor._layout_params["scale"]


class QuIPHadamardINT8Layout(QuantizedLayout):
    """Transformed-space QuIP weight ``Q' [N_pad, K_pad]`` with per-row scale
    ``[N_pad]`` and sign vectors (written by ``store_transformed``,
    converters/quip_int8.py:1558-1608, quantization.py:651-662).

    ``linear(x, W) = (FWHT(FWHT(pad(x) * sign_col) @ (scale * Q')^T) * sign_row)[:, :N] + bias``
    """

    @classmethod
    def quantize(cls, tensor, scale=None, sign_row=None, sign_col=None, **kwargs):
        raise NotImplementedError("use converters.quip_int8.QuIPInt8Converter(store_transformed=True)")

    @staticmethod
    def dequantize(qdata, scale, sign_row, sign_col, out_features, in_features, orig_dtype, **kwargs):
        # W = diag(s_u) H (scale * Q') H diag(s_v), sliced
        w = ops.dequant(qdata, scale.reshape(-1), L.QI8_S_ROW, 0, torch.float32)
        from .hadamard_kernels import fast_hadamard_transform
        w = fast_hadamard_transform(w)
        w = fast_hadamard_transform(w.t().contiguous()).t()
        w = w * sign_row.view(-1, 1) * sign_col.view(1, -1)
        return w[:out_features, :in_features].to(orig_dtype)

    @classmethod
    def get_plain_tensors(cls, qtensor):
        p = qtensor._layout_params
        return qtensor._qdata, p["scale"], p["sign_row"], p["sign_col"]


QUANT_ALGOS = {
    "int8_blockwise": {
        "storage_t": torch.int8,
        "required_parameters": {"weight_scale"},
        "optional_parameters": {"input_scale"},
        "comfy_tensor_layout": "BlockWiseINT8Layout",
        "group_size": 128,
        "asymmetric_layout": True,
    },
}

LAYOUTS = {
    "BlockWiseINT8Layout": BlockWiseINT8Layout,
    "TensorWiseINT8Layout": TensorWiseINT8Layout,
    "AxisWiseINT8Layout": AxisWiseINT8Layout,
    "QuIPHadamardINT8Layout": QuIPHadamardINT8Layout,
}


# ------------------------------------------------------------- handlers
def _int8_gemm_or_fallback(a_int8, a_scale, b_int8, b_scale, block_size, bias=None, out_quant=False,
                           out_dtype=torch.bfloat16):
    """Block-scaled GEMM (comfy/quant_ops.py:358-371) on the tcgen05 kernel;
    with ``out_quant`` the epilogue requantizes the output per (row, block)
    (the reference's int8_gemm_quant / int8_addmm_quant)."""
    K, batch, N = a_int8.shape[-1], a_int8.shape[:-1], b_int8.shape[0]
    a2 = a_int8.reshape(-1, K).contiguous()
    a_s2 = a_scale.reshape(-1, a_scale.shape[-1]).contiguous()
    if out_quant:
        q, s = ops.gemm_i8_quant(a2, b_int8.contiguous(), a_s2, b_scale.contiguous(), bias, block_size)
        return q.reshape(*batch, N), s.reshape(*batch, N // block_size)
    b_kind = ops.scale_kind(b_scale, N, K, True, block_size)
    res = ops.gemm_i8(a2, b_int8.contiguous(), a_s2, L.QI8_S_ROW_KBLOCK, b_scale.contiguous(), b_kind, bias,
                      out_dtype)
    return res.reshape(*batch, N)


def _linear_w8a8_token(x, w_q, w_s, w_kind, bias, out_dtype, act=L.QI8_ACT_NONE):
    """Per-token activation quantization + int8 GEMM with the fused epilogue."""
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    x_q, x_s = ops.quant_rows(x2, L.QI8_Q_TOKEN)
    y = ops.gemm_i8(x_q, w_q, x_s, L.QI8_S_ROW, w_s, w_kind, bias, out_dtype, act)
    return y.reshape(*x.shape[:-1], w_q.shape[0])


@register_layout_op(torch.ops.aten.linear.default, "BlockWiseINT8Layout")
def int8_linear(func, args, kwargs):
    x, weight = args[0], args[1]
    bias = args[2] if len(args) > 2 else None
    if isinstance(x, QuantizedTensor) and isinstance(weight, QuantizedTensor):
        a_int8, a_scale, a_bs, _ = BlockWiseINT8Layout.get_plain_tensors(x)
        b_int8, b_scale, b_bs, _ = BlockWiseINT8Layout.get_plain_tensors(weight)
        out_dtype = kwargs.get("out_dtype", x._layout_params["orig_dtype"])
        out_quant = kwargs.get("out_quant", False)
        res = _int8_gemm_or_fallback(a_int8, a_scale, b_int8, b_scale, a_bs, bias, out_quant, out_dtype)
        if out_quant:
            return QuantizedTensor(res[0], "BlockWiseINT8Layout",
                                   {"scale": res[1], "block_size": a_bs, "is_weight": False, "orig_dtype": out_dtype})
        return res.to(out_dtype)
    if isinstance(weight, QuantizedTensor) and not isinstance(x, QuantizedTensor):
        b_int8, b_scale, b_bs, _ = BlockWiseINT8Layout.get_plain_tensors(weight)
        N, K = b_int8.shape
        if b_scale.numel() == N * (K // b_bs) and b_scale.numel() != (N // b_bs) * (K // b_bs):
            # QuIP block-requant weight: W8A8 with per-token activations
            return _linear_w8a8_token(x, b_int8, b_scale.reshape(N, -1), L.QI8_S_ROW_KBLOCK, bias,
                                      kwargs.get("out_dtype", x.dtype))
    return torch.nn.functional.linear(x.dequantize() if isinstance(x, QuantizedTensor) else x,
                                      weight.dequantize() if isinstance(weight, QuantizedTensor) else weight, bias)


@register_layout_op(torch.ops.aten.mm.default, "BlockWiseINT8Layout")
def int8_mm(func, args, kwargs):
    x, weight = args[0], args[1]
    if isinstance(x, QuantizedTensor) and isinstance(weight, QuantizedTensor):
        a_int8, a_scale, a_bs, _ = BlockWiseINT8Layout.get_plain_tensors(x)
        b_int8, b_scale, b_bs, _ = BlockWiseINT8Layout.get_plain_tensors(weight)
        out_dtype = kwargs.get("out_dtype", x._layout_params["orig_dtype"])
        out_quant = kwargs.get("out_quant", False)
        K = a_int8.shape[-1]
        if b_int8.shape[0] == K and b_int8.shape[1] != K:
            b_int8, b_scale = b_int8.t().contiguous(), b_scale.t().contiguous()
        res = _int8_gemm_or_fallback(a_int8, a_scale, b_int8, b_scale, a_bs, None, out_quant, out_dtype)
        if out_quant:
            return QuantizedTensor(res[0], "BlockWiseINT8Layout",
                                   {"scale": res[1], "block_size": a_bs, "is_weight": False, "orig_dtype": out_dtype})
        return res.to(out_dtype)
    return func(args[0].dequantize() if isinstance(args[0], QuantizedTensor) else args[0],
                args[1].dequantize() if isinstance(args[1], QuantizedTensor) else args[1])


@register_layout_op(torch.ops.aten.addmm.default, "BlockWiseINT8Layout")
def int8_addmm(func, args, kwargs):
    bias, x, weight = args[0], args[1], args[2]
    if isinstance(x, QuantizedTensor) and isinstance(weight, QuantizedTensor):
        a_int8, a_scale, a_bs, _ = BlockWiseINT8Layout.get_plain_tensors(x)
        b_int8, b_scale, b_bs, _ = BlockWiseINT8Layout.get_plain_tensors(weight)
        out_dtype = kwargs.get("out_dtype", x._layout_params["orig_dtype"])
        out_quant = kwargs.get("out_quant", False)
        K = a_int8.shape[-1]
        if b_int8.shape[0] == K:
            b_int8, b_scale = b_int8.t().contiguous(), b_scale.t().contiguous()
        res = _int8_gemm_or_fallback(a_int8, a_scale, b_int8, b_scale, a_bs, bias, out_quant, out_dtype)
        if out_quant:
            return QuantizedTensor(res[0], "BlockWiseINT8Layout",
                                   {"scale": res[1], "block_size": a_bs, "is_weight": False, "orig_dtype": out_dtype})
        return res.to(out_dtype)
    deq = [a.dequantize() if isinstance(a, QuantizedTensor) else a for a in args[:3]]
    return func(*deq, **kwargs)


@register_layout_op(torch.ops.aten.view.default, "BlockWiseINT8Layout")
def int8_view(func, args, kwargs):
    x = args[0]
    if isinstance(x, QuantizedTensor):
        return QuantizedTensor(func(x._qdata, *args[1:], **kwargs), "BlockWiseINT8Layout", x._layout_params)
    return func(*args, **kwargs)


@register_layout_op(torch.ops.aten.t.default, "BlockWiseINT8Layout")
def int8_transpose(func, args, kwargs):
    x = args[0]
    if isinstance(x, QuantizedTensor):
        params = dict(x._layout_params)
        if params.get("is_weight"):
            params["scale"] = params["scale"].t().contiguous()
        return QuantizedTensor(func(x._qdata, *args[1:], **kwargs), "BlockWiseINT8Layout", params)
    return func(*args, **kwargs)


@register_layout_op(torch.ops.aten.gelu.default, "BlockWiseINT8Layout")
def int8_gelu(func, args, kwargs):
    x = args[0]
    if isinstance(x, QuantizedTensor):
        from .int8_kernels import int8_gelu as k_gelu
        qdata, scale, bs, _ = BlockWiseINT8Layout.get_plain_tensors(x)
        q, s = k_gelu(qdata, scale, block_size=bs)
        return QuantizedTensor(q, "BlockWiseINT8Layout", {"scale": s.to(torch.float32), "block_size": bs,
                                                          "is_weight": False,
                                                          "orig_dtype": x._layout_params["orig_dtype"]})
    return func(*args, **kwargs)


@register_layout_op(torch.ops.aten.add_.Tensor, "BlockWiseINT8Layout")
def int8_add_(func, args, kwargs):
    target = args[0]
    if isinstance(target, QuantizedTensor) and target._layout_params.get("is_weight"):
        other = args[1].dequantize() if isinstance(args[1], QuantizedTensor) else args[1]
        res = target.dequantize() + other
        q, params = BlockWiseINT8Layout.quantize(res, block_size=target._layout_params["block_size"], is_weight=True)
        target._qdata.copy_(q)
        target._layout_params["scale"].copy_(params["scale"])
        return target
    return QuantizedTensor._dequant_and_fallback(func, args, kwargs)


@register_layout_op(torch.ops.aten.linear.default, "TensorWiseINT8Layout")
@register_layout_op(torch.ops.aten.linear.default, "AxisWiseINT8Layout")
def optimized_linear(func, args, kwargs):
    """W8A8 linear (comfy/quant_ops.py:461-475): per-token act quant, int8 GEMM,
    ``acc * (x_s * w_s) + bias`` -> input dtype, fused in one epilogue."""
    x, weight = args[0], args[1]
    bias = args[2] if len(args) > 2 else None
    if isinstance(weight, QuantizedTensor) and not isinstance(x, QuantizedTensor):
        w_q, w_s = LAYOUTS[weight.layout_type].get_plain_tensors(weight)
        N = w_q.shape[0]
        kind = L.QI8_S_SCALAR if w_s.numel() == 1 else L.QI8_S_ROW
        assert kind == L.QI8_S_SCALAR or w_s.numel() == N, f"weight scale of shape {tuple(w_s.shape)}"
        return _linear_w8a8_token(x, w_q, w_s.reshape(-1) if kind == L.QI8_S_ROW else w_s, kind, bias, x.dtype)
    return QuantizedTensor._dequant_and_fallback(func, args, kwargs)


@register_layout_op(torch.ops.aten.linear.default, "QuIPHadamardINT8Layout")
def quip_hadamard_linear(func, args, kwargs):
    """Transformed-space W8A8 linear: K1 (sign + FWHT + per-token int8), K2
    (tcgen05 GEMM, fp32 ``x_s * w_s`` epilogue), K3 (FWHT + sign + slice + bias)."""
    x, weight = args[0], args[1]
    bias = args[2] if len(args) > 2 else None
    if not isinstance(weight, QuantizedTensor) or isinstance(x, QuantizedTensor):
        return QuantizedTensor._dequant_and_fallback(func, args, kwargs)
    q, scale, s_u, s_v = QuIPHadamardINT8Layout.get_plain_tensors(weight)
    p = weight._layout_params
    N, K = p["out_features"], p["in_features"]
    N_pad, K_pad = q.shape
    assert x.shape[-1] == K, f"input has {x.shape[-1]} features, weight expects {K}"
    x2 = x.reshape(-1, K)
    xq, xs = ops.rotate_quant_rows(x2, s_v, K_pad)
    y_had = ops.gemm_i8(xq, q, xs, L.QI8_S_ROW, scale.reshape(-1), L.QI8_S_ROW, None, torch.float32)
    y = ops.unrotate_rows(y_had, s_u, N, bias, x.dtype)
    return y.reshape(*x.shape[:-1], N)


def quip_hadamard_weight(q_rot: torch.Tensor, scale: torch.Tensor, sign_row: torch.Tensor, sign_col: torch.Tensor,
                         out_features: int, in_features: int, orig_dtype=torch.bfloat16) -> QuantizedTensor:
    """Builds a ``QuIPHadamardINT8Layout`` weight from a transformed-space
    checkpoint entry (``weight``, ``weight_scale``, ``sign_row``, ``sign_col``)."""
    params = {"scale": scale.reshape(-1).to(torch.float32).contiguous(),
              "sign_row": sign_row.to(torch.float32).contiguous(),
              "sign_col": sign_col.to(torch.float32).contiguous(),
              "out_features": int(out_features), "in_features": int(in_features), "orig_dtype": orig_dtype}
    return QuantizedTensor(q_rot.contiguous(), "QuIPHadamardINT8Layout", params)


logging.getLogger(__name__).debug("qi8 comfy quant_ops loaded")
