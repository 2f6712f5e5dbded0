"""torch-facing wrappers of the libqi8 kernels.

Outputs are allocated here with the PyTorch caching allocator (the C library
never allocates); every launch goes on ``torch.cuda.current_stream()``.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import torch

from . import _lib as L


def _next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def _rows2d(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def _sign(s: Optional[torch.Tensor], n: int, device) -> Optional[torch.Tensor]:
    if s is None:
        return None
    s = s.to(device=device, dtype=torch.float32).contiguous().reshape(-1)
    assert s.numel() == n, f"sign vector has {s.numel()} entries, expected {n}"
    return s


def quant_rows(x: torch.Tensor, mode: int = L.QI8_Q_TOKEN, block: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-token (mode TOKEN) or per-128-block (mode BLOCK) int8 quantization of
    the last dimension.  Returns ``(q int8 [..., n], scale fp32 [...] or [..., n/128])``."""
    L.require_cuda(x)
    x2 = _rows2d(x)
    rows, n = x2.shape
    q = torch.empty((rows, n), dtype=torch.int8, device=x.device)
    base_mode = mode & 0xFF
    ns = 1 if base_mode == L.QI8_Q_TOKEN else n // block
    s = torch.empty((rows, ns), dtype=torch.float32, device=x.device)
    lib = L.load()
    L.check(lib.qi8_quant_rows(L.ptr(x2), L.dtype_code(x2.dtype), rows, n, x2.stride(0), mode, block,
                               L.ptr(q), n, L.ptr(s), L.stream_ptr(x.device)), "qi8_quant_rows")
    q = q.reshape(x.shape)
    if base_mode == L.QI8_Q_TOKEN:
        return q, s.reshape(*x.shape[:-1], 1)
    return q, s.reshape(*x.shape[:-1], ns)


def rotate_quant_rows(x: torch.Tensor, sign: Optional[torch.Tensor], n_pad: Optional[int] = None,
                      normalize: bool = True, mode: int = L.QI8_Q_TOKEN) -> Tuple[torch.Tensor, torch.Tensor]:
    """K1: ``quant(FWHT(pad(x, n_pad) * sign))``.  Returns ``(q [rows, n_pad], scale)``."""
    L.require_cuda(x)
    x2 = _rows2d(x)
    rows, n = x2.shape
    n_pad = n_pad or _next_pow2(n)
    if n_pad & (n_pad - 1):
        raise ValueError(f"Last dimension must be a power of 2, got {n_pad}")
    q = torch.empty((rows, n_pad), dtype=torch.int8, device=x.device)
    ns = 1 if mode == L.QI8_Q_TOKEN else n_pad // 128
    s = torch.empty((rows, ns), dtype=torch.float32, device=x.device)
    sg = _sign(sign, n_pad, x.device)
    lib = L.load()
    L.check(lib.qi8_rotate_quant_rows(L.ptr(x2), L.dtype_code(x2.dtype), rows, n, x2.stride(0), n_pad,
                                      L.ptr(sg), int(normalize), mode, L.ptr(q), L.ptr(s),
                                      L.stream_ptr(x.device)), "qi8_rotate_quant_rows")
    return q, s


def fwht_rows(x: torch.Tensor, n_pad: Optional[int] = None, pre_sign: Optional[torch.Tensor] = None,
              post_sign: Optional[torch.Tensor] = None, normalize: bool = True,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FWHT of every row (last dim) to fp32 ``[..., n_pad]``."""
    L.require_cuda(x)
    x2 = _rows2d(x)
    rows, n = x2.shape
    n_pad = n_pad or n
    if n_pad & (n_pad - 1) or n_pad < 1:
        raise ValueError(f"Last dimension must be a power of 2, got {n_pad}")
    if out is None:
        out = torch.empty((rows, n_pad), dtype=torch.float32, device=x.device)
    lib = L.load()
    L.check(lib.qi8_fwht_rows(L.ptr(x2), L.dtype_code(x2.dtype), rows, n, x2.stride(0), n_pad,
                              L.ptr(_sign(pre_sign, n_pad, x.device)), L.ptr(_sign(post_sign, n_pad, x.device)),
                              int(normalize), L.ptr(out), L.stream_ptr(x.device)), "qi8_fwht_rows")
    return out.reshape(*x.shape[:-1], n_pad)


def fwht_cols_(x: torch.Tensor, final_mode: int = 0, factor: float = 1.0) -> torch.Tensor:
    """In-place FWHT down the columns of a contiguous fp32 matrix ``[rows, cols]``."""
    L.require_cuda(x)
    assert x.dtype == torch.float32 and x.dim() == 2 and x.stride(1) == 1, "x must be a row-major fp32 matrix"
    rows, cols = x.shape
    if rows & (rows - 1):
        raise ValueError(f"Second-to-last dimension must be power of 2, got {rows}")
    lib = L.load()
    L.check(lib.qi8_fwht_cols(L.ptr(x), rows, cols, x.stride(0), final_mode, float(factor),
                              L.stream_ptr(x.device)), "qi8_fwht_cols")
    return x


def unrotate_rows(y_had: torch.Tensor, sign_u: Optional[torch.Tensor], n_out: int,
                  bias: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """K3: ``(FWHT(y_had) * sign_u)[:, :n_out] + bias`` -> ``out_dtype``."""
    L.require_cuda(y_had)
    assert y_had.dtype == torch.float32 and y_had.is_contiguous(), "y_had must be contiguous fp32"
    rows, n_pad = y_had.reshape(-1, y_had.shape[-1]).shape
    out = torch.empty((rows, n_out), dtype=out_dtype, device=y_had.device)
    b = None if bias is None else bias.contiguous()
    lib = L.load()
    L.check(lib.qi8_unrotate_rows(L.ptr(y_had), rows, n_pad, L.ptr(_sign(sign_u, n_pad, y_had.device)),
                                  L.ptr(b), L.dtype_code(b.dtype) if b is not None else 0, n_out, L.ptr(out),
                                  L.dtype_code(out_dtype), n_out, L.stream_ptr(y_had.device)),
            "qi8_unrotate_rows")
    return out


def scale_kind(scale: Optional[torch.Tensor], rows: int, K: int, is_weight: bool, block: int = 128) -> int:
    """Classify a scale tensor for ``gemm_i8`` by its element count."""
    if scale is None:
        return L.QI8_S_NONE
    n = scale.numel()
    kb = K // block
    if n == 1 and not (rows == 1 and kb == 1 and scale.dim() >= 2):
        return L.QI8_S_SCALAR
    if n == rows:
        return L.QI8_S_ROW
    if n == rows * kb:
        return L.QI8_S_ROW_KBLOCK
    if is_weight and n == ((rows + block - 1) // block) * kb:
        return L.QI8_S_TILE128
    raise AssertionError(f"cannot interpret scale of shape {tuple(scale.shape)} for rows={rows}, K={K}")


def gemm_i8(a: torch.Tensor, b: torch.Tensor, a_scale: Optional[torch.Tensor] = None, a_kind: Optional[int] = None,
            b_scale: Optional[torch.Tensor] = None, b_kind: Optional[int] = None,
            bias: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16,
            act: int = L.QI8_ACT_NONE, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """K2: ``a [M, K] int8 . b [N, K]^T int8`` with the fused epilogue."""
    L.require_cuda(a, b)
    assert a.dtype == torch.int8 and b.dtype == torch.int8, "int8 operands required"
    a2 = a.reshape(-1, a.shape[-1])
    assert a2.is_contiguous() and b.is_contiguous() and b.dim() == 2, "Input tensors must be contiguous"
    M, K = a2.shape
    N = b.shape[0]
    assert b.shape[1] == K, f"Shape mismatch: b.shape={tuple(b.shape)}, expected [N, {K}]"
    if a_scale is not None:
        a_scale = a_scale.to(torch.float32).contiguous()
        a_kind = scale_kind(a_scale, M, K, False) if a_kind is None else a_kind
    else:
        a_kind = L.QI8_S_NONE
    if b_scale is not None:
        b_scale = b_scale.to(torch.float32).contiguous()
        b_kind = scale_kind(b_scale, N, K, True) if b_kind is None else b_kind
    else:
        b_kind = L.QI8_S_NONE
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    bb = None if bias is None else bias.contiguous()
    lib = L.load()
    # small output grids split K (int32 partials in a workspace, identical results)
    ws_bytes = _gemm_ws_bytes(M, N, K, a_kind, b_kind)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=a.device) if ws_bytes else None
    L.check(lib.qi8_gemm_i8_ws(L.ptr(a2), L.ptr(b), M, N, K, L.ptr(a_scale), a_kind, L.ptr(b_scale), b_kind,
                               L.ptr(bb), L.dtype_code(bb.dtype) if bb is not None else 0, L.ptr(out),
                               L.dtype_code(out.dtype), out.stride(0), act, L.ptr(ws), ws_bytes,
                               L.stream_ptr(a.device)), "qi8_gemm_i8")
    return out.reshape(*a.shape[:-1], N)


def gemm_i8_quant(a: torch.Tensor, b: torch.Tensor, a_scale: torch.Tensor, b_scale: torch.Tensor,
                  bias: Optional[torch.Tensor] = None, out_block: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """K2 with the output requantized per (row, 128-column block) in the
    epilogue: ``a [..., K]`` int8 with block scales ``[..., K/128]``, ``b [N, K]``
    with ``[N/128, K/128]`` tile or ``[N, K/128]`` row-block scales.  Returns
    ``(q int8 [..., N], scale fp32 [..., N/128])``."""
    L.require_cuda(a, b)
    assert a.dtype == torch.int8 and b.dtype == torch.int8, "int8 operands required"
    a2 = a.reshape(-1, a.shape[-1])
    assert a2.is_contiguous() and b.is_contiguous() and b.dim() == 2, "Input tensors must be contiguous"
    M, K = a2.shape
    N = b.shape[0]
    assert b.shape[1] == K, f"Shape mismatch: b.shape={tuple(b.shape)}, expected [N, {K}]"
    assert N % out_block == 0, f"N={N} must be divisible by out_block_size={out_block}"
    a_scale = a_scale.to(torch.float32).contiguous()
    b_scale = b_scale.to(torch.float32).contiguous()
    assert a_scale.numel() == M * (K // 128), f"activation scales of shape {tuple(a_scale.shape)}"
    b_kind = L.QI8_S_ROW_KBLOCK if b_scale.numel() == N * (K // 128) else scale_kind(b_scale, N, K, True)
    q = torch.empty((M, N), dtype=torch.int8, device=a.device)
    s = torch.empty((M, N // out_block), dtype=torch.float32, device=a.device)
    bb = None if bias is None else bias.contiguous()
    L.check(L.load().qi8_gemm_i8_quant(L.ptr(a2), L.ptr(b), M, N, K, L.ptr(a_scale), L.QI8_S_ROW_KBLOCK,
                                       L.ptr(b_scale), b_kind, L.ptr(bb), L.dtype_code(bb.dtype) if bb is not None else 0,
                                       L.ptr(q), N, L.ptr(s), out_block, L.stream_ptr(a.device)), "qi8_gemm_i8_quant")
    return q.reshape(*a.shape[:-1], N), s.reshape(*a.shape[:-1], N // out_block)


def int8_gelu(q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """GELU of a block-quantized int8 activation, requantized per block."""
    L.require_cuda(q, scale)
    assert q.dtype == torch.int8 and q.is_contiguous() and scale.is_contiguous(), "Input tensors must be contiguous"
    n = q.shape[-1]
    rows = q.numel() // n
    q_out = torch.empty_like(q)
    s_out = torch.empty(scale.shape, dtype=torch.float32, device=q.device)
    L.check(L.load().qi8_int8_gelu(L.ptr(q), L.ptr(scale.to(torch.float32)), rows, n, block, L.ptr(q_out),
                                   L.ptr(s_out), L.stream_ptr(q.device)), "qi8_int8_gelu")
    return q_out, s_out


_WS_CACHE = {}


def _gemm_ws_bytes(M: int, N: int, K: int, a_kind: int, b_kind: int) -> int:
    key = (torch.cuda.current_device(), M, N, K, a_kind, b_kind)
    v = _WS_CACHE.get(key)
    if v is None:
        v = _WS_CACHE[key] = int(L.load().qi8_gemm_workspace_bytes(M, N, K, a_kind, b_kind))
    return v


def dequant(q: torch.Tensor, scale: torch.Tensor, kind: int, block: int = 128,
            out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    L.require_cuda(q, scale)
    q2 = q.reshape(-1, q.shape[-1]).contiguous()
    rows, n = q2.shape
    out = torch.empty((rows, n), dtype=out_dtype, device=q.device)
    lib = L.load()
    L.check(lib.qi8_dequant(L.ptr(q2), rows, n, L.ptr(scale.to(torch.float32).contiguous()), kind, block,
                            L.ptr(out), L.dtype_code(out_dtype), L.stream_ptr(q.device)), "qi8_dequant")
    return out.reshape(q.shape)


def quant_weight(w: torch.Tensor, kind: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Tensorwise (SCALAR), per-row (ROW) or Triton-style 128x128 tile (TILE128) weight quantization."""
    L.require_cuda(w)
    w2 = w.reshape(-1, w.shape[-1]).contiguous()
    rows, n = w2.shape
    q = torch.empty((rows, n), dtype=torch.int8, device=w.device)
    if kind == L.QI8_S_SCALAR:
        s = torch.empty((), dtype=torch.float32, device=w.device)
    elif kind == L.QI8_S_ROW:
        s = torch.empty((rows, 1), dtype=torch.float32, device=w.device)
    else:
        s = torch.empty((rows // 128, n // 128), dtype=torch.float32, device=w.device)
    ws = torch.empty(64, dtype=torch.uint8, device=w.device)
    lib = L.load()
    L.check(lib.qi8_quant_weight(L.ptr(w2), L.dtype_code(w2.dtype), rows, n, kind, L.ptr(q), L.ptr(s), L.ptr(ws),
                                 ws.numel(), L.stream_ptr(w.device)), "qi8_quant_weight")
    return q.reshape(w.shape), s


def quip_workspace_bytes(M: int, N: int) -> int:
    return int(L.load().qi8_quip_workspace_bytes(M, N))


def quip_convert(w: torch.Tensor, s_u: torch.Tensor, s_v: torch.Tensor, store_transformed: bool = False,
                 requant: int = L.QI8_REQ_ROW, block: int = 128, want_dequant: bool = True,
                 workspace: Optional[torch.Tensor] = None):
    """K4: QuIP Hadamard conversion of one weight.  Returns ``(q, scale, dequantized_weight or None)``."""
    L.require_cuda(w)
    assert w.dim() == 2, "weight must be 2-D"
    w = w.contiguous()
    M, N = w.shape
    Mp, Np = _next_pow2(M), _next_pow2(N)
    su = _sign(s_u, Mp, w.device)
    sv = _sign(s_v, Np, w.device)
    nbytes = quip_workspace_bytes(M, N)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
    if store_transformed:
        q = torch.empty((Mp, Np), dtype=torch.int8, device=w.device)
        s = torch.empty((Mp, 1), dtype=torch.float32, device=w.device)
    else:
        q = torch.empty((M, N), dtype=torch.int8, device=w.device)
        if requant == L.QI8_REQ_BLOCK and N % block == 0:
            s = torch.empty((M, N // block, 1), dtype=torch.float32, device=w.device)
        elif requant == L.QI8_REQ_GLOBAL:
            s = torch.empty((), dtype=torch.float32, device=w.device)
        else:
            s = torch.empty((M, 1), dtype=torch.float32, device=w.device)
    deq = torch.empty((M, N), dtype=torch.float32, device=w.device) if want_dequant else None
    lib = L.load()
    L.check(lib.qi8_quip_convert(L.ptr(w), L.dtype_code(w.dtype), M, N, L.ptr(su), L.ptr(sv), int(store_transformed),
                                 requant, block, L.ptr(q), L.ptr(s), L.ptr(deq), L.ptr(workspace), workspace.numel(),
                                 L.stream_ptr(w.device)), "qi8_quip_convert")
    return q, s, deq


def weight_rotate2d(w: torch.Tensor, s_u: torch.Tensor, s_v: torch.Tensor, inverse: bool = False,
                    shape: Optional[tuple] = None) -> torch.Tensor:
    """Two-sided signed Hadamard rotation of a weight (the converter's
    incoherence step, converters/quip_int8.py:523-551 / :1489-1506).

    Forward: ``w`` [M, N] -> fp32 [M_pad, N_pad] = FHT_N(FHT_M(pad(w) s_u s_v^T)).
    Inverse: ``w`` [M_pad, N_pad] -> fp32 ``shape`` (default [M_pad, N_pad]) =
    slice(FHT_M(FHT_N(w)) s_u s_v^T).  Pads are ``len(s_u)``, ``len(s_v)``.
    """
    L.require_cuda(w)
    assert w.dim() == 2, "weight must be 2-D"
    w = w.contiguous()
    Mp, Np = int(s_u.numel()), int(s_v.numel())
    su = _sign(s_u, Mp, w.device)
    sv = _sign(s_v, Np, w.device)
    lib = L.load()
    if not inverse:
        M, N = w.shape
        out = torch.empty((Mp, Np), dtype=torch.float32, device=w.device)
        ws, nws = None, 0
    else:
        assert tuple(w.shape) == (Mp, Np), f"inverse rotation takes a [{Mp}, {Np}] matrix, got {tuple(w.shape)}"
        M, N = shape if shape is not None else (Mp, Np)
        out = torch.empty((M, N), dtype=torch.float32, device=w.device)
        ws = torch.empty((Mp, Np), dtype=torch.float32, device=w.device)
        nws = ws.numel() * 4
    L.check(lib.qi8_weight_rotate2d(L.ptr(w), L.dtype_code(w.dtype), M, N, Mp, Np, L.ptr(su), L.ptr(sv),
                                    int(bool(inverse)), L.ptr(out), L.ptr(ws), nws, L.stream_ptr(w.device)),
            "qi8_weight_rotate2d")
    return out


def allgather_cols(y_local: torch.Tensor, nccl_comm: int, world: int,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather of column shards ``[T, n_loc]`` into ``[T, world * n_loc]``
    over a caller-created NCCL communicator (``ncclComm_t`` as an integer)."""
    L.require_cuda(y_local)
    y_local = y_local.contiguous()
    T, n_loc = y_local.shape
    if out is None:
        out = torch.empty((T, world * n_loc), dtype=y_local.dtype, device=y_local.device)
    scratch = torch.empty((world, T, n_loc), dtype=y_local.dtype, device=y_local.device)
    lib = L.load()
    L.check(lib.qi8_allgather_cols(L.ptr(y_local), L.dtype_code(y_local.dtype), T, n_loc, L.ptr(out), out.stride(0),
                                   ctypes.c_void_p(nccl_comm), L.ptr(scratch), scratch.numel() * scratch.element_size(),
                                   L.stream_ptr(y_local.device)), "qi8_allgather_cols")
    return out


def gather_layout(gathered: torch.Tensor, world: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``[world, T, n_loc]`` (or ``[world * T, n_loc]``) all-gather result ->
    ``[T, world * n_loc]``; ``out`` may be a row-strided view."""
    L.require_cuda(gathered)
    assert gathered.is_contiguous(), "gathered must be contiguous"
    n_loc = gathered.shape[-1]
    T = gathered.numel() // (world * n_loc)
    if out is None:
        out = torch.empty((T, world * n_loc), dtype=gathered.dtype, device=gathered.device)
    assert out.shape == (T, world * n_loc) and out.stride(1) == 1, "out must be [T, world * n_loc] row-major"
    L.check(L.load().qi8_gather_layout(L.ptr(gathered), L.dtype_code(gathered.dtype), world, T, n_loc, L.ptr(out),
                                       out.stride(0), L.stream_ptr(gathered.device)), "qi8_gather_layout")
    return out


def requant_weight(w: torch.Tensor, requant: int = L.QI8_REQ_ROW, block: int = 128):
    """QuIP requant rule without rotation (converters/quip_int8.py:1614-1669)."""
    L.require_cuda(w)
    assert w.dim() == 2 and w.stride(1) == 1, "weight must be a row-major 2-D tensor"
    M, N = w.shape
    q = torch.empty((M, N), dtype=torch.int8, device=w.device)
    if requant == L.QI8_REQ_BLOCK and N % block == 0:
        s = torch.empty((M, N // block, 1), dtype=torch.float32, device=w.device)
    elif requant == L.QI8_REQ_GLOBAL:
        s = torch.empty((), dtype=torch.float32, device=w.device)
    else:
        s = torch.empty((M, 1), dtype=torch.float32, device=w.device)
    ws = torch.empty(64, dtype=torch.uint8, device=w.device)
    lib = L.load()
    L.check(lib.qi8_requant_weight(L.ptr(w), L.dtype_code(w.dtype), M, N, w.stride(0), requant, block, L.ptr(q),
                                   L.ptr(s), L.ptr(ws), ws.numel(), L.stream_ptr(w.device)), "qi8_requant_weight")
    return q, s


# ---------------------------------------------------------------------------
# QuIP with the reference's defaults (diagonal rescaling, random permutation,
# damping, act-order, fp64 Hessian factorization, blocked LDLQ)
# ---------------------------------------------------------------------------

def col_sumsq(w: torch.Tensor) -> torch.Tensor:
    """``(W ** 2).sum(dim=0)`` in fp32, summed in torch's CPU order
    (converters/quip_int8.py:266)."""
    L.require_cuda(w)
    assert w.dim() == 2 and w.stride(1) == 1, "weight must be a row-major 2-D tensor"
    M, N = w.shape
    out = torch.empty(N, dtype=torch.float32, device=w.device)
    L.check(L.load().qi8_col_sumsq(L.ptr(w), L.dtype_code(w.dtype), M, N, w.stride(0), L.ptr(out),
                                   L.stream_ptr(w.device)), "qi8_col_sumsq")
    return out


def scale2d(x: Optional[torch.Tensor], shape: tuple, row: Optional[torch.Tensor] = None,
            col: Optional[torch.Tensor] = None, divide: bool = False, device=None) -> torch.Tensor:
    """``(x * col[None, :]) * row[:, None]`` or ``x / col[None, :]`` in fp32
    (converters/quip_int8.py:280-285, 303); ``x=None`` is the identity."""
    dev = x.device if x is not None else device
    if x is not None:
        L.require_cuda(x)
        assert x.stride(1) == 1, "x must be row-major"
    M, N = shape
    out = torch.empty((M, N), dtype=torch.float32, device=dev)
    L.check(L.load().qi8_scale2d(L.ptr(x), L.dtype_code(x.dtype) if x is not None else 0, M, N,
                                 x.stride(0) if x is not None else N, L.ptr(row), L.ptr(col), int(bool(divide)),
                                 L.ptr(out), N, L.stream_ptr(dev)), "qi8_scale2d")
    return out


def ldlq_prepare(w_rot: torch.Tensor, h_rot: torch.Tensor, cols: torch.Tensor, dead: torch.Tensor,
                 diag: torch.Tensor):
    """Gather W' and H' into LDLQ column order ``cols`` (dead columns zeroed,
    damped diagonal ``diag``), the per-row scale, and the Hessian reversed
    for the factorization.  Returns ``(W_p fp32 [M, N], scale [M, 1], H_rev fp64 [N, N])``."""
    M, N = w_rot.shape
    dev = w_rot.device
    wp = torch.empty((M, N), dtype=torch.float32, device=dev)
    sc = torch.empty((M, 1), dtype=torch.float32, device=dev)
    hrev = torch.empty((N, N), dtype=torch.float64, device=dev)
    L.check(L.load().qi8_ldlq_prepare(L.ptr(w_rot), L.ptr(h_rot), M, N, L.ptr(cols), L.ptr(dead), L.ptr(diag),
                                      L.ptr(wp), L.ptr(sc), L.ptr(hrev), L.stream_ptr(dev)), "qi8_ldlq_prepare")
    return wp, sc, hrev


def hinv_upper(h_rev: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Upper Cholesky factor of H^-1 from the reversed damped Hessian (fp64,
    overwritten); returns ``(U fp32 [N, N], info int32 device scalar)`` --
    info != 0 marks a non-positive pivot (the reference then uses the
    identity, converters/quip_int8.py:1211-1216)."""
    N = h_rev.shape[0]
    dev = h_rev.device
    lib = L.load()
    hinv = torch.empty((N, N), dtype=torch.float32, device=dev)
    info = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.empty(int(lib.qi8_hinv_workspace_bytes(N)), dtype=torch.uint8, device=dev)
    L.check(lib.qi8_hinv_upper(L.ptr(h_rev), N, L.ptr(hinv), L.ptr(info), L.ptr(ws), ws.numel(),
                               L.stream_ptr(dev)), "qi8_hinv_upper")
    return hinv, info


def eye_f32(n: int, device) -> torch.Tensor:
    out = torch.empty((n, n), dtype=torch.float32, device=device)
    L.check(L.load().qi8_eye_f32(L.ptr(out), n, L.stream_ptr(device)), "qi8_eye_f32")
    return out


def ldlq(w: torch.Tensor, hinv: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    """The LDLQ pass (converters/quip_int8.py:813-945); ``w`` fp32 [M, N] is
    consumed (updated in place).  Returns ``Q'`` int8 [M, N]."""
    M, N = w.shape
    dev = w.device
    lib = L.load()
    q = torch.empty((M, N), dtype=torch.int8, device=dev)
    ws = torch.empty(int(lib.qi8_ldlq_workspace_bytes(M, N, block)), dtype=torch.uint8, device=dev)
    L.check(lib.qi8_ldlq(L.ptr(w), M, N, L.ptr(hinv), L.ptr(scale), block, L.ptr(q), L.ptr(ws), ws.numel(),
                         L.stream_ptr(dev)), "qi8_ldlq")
    return q


def ldlq_finish(q: torch.Tensor, scale: torch.Tensor, cols: torch.Tensor, want_deq: bool = True,
                want_q: bool = False):
    """Scatter LDLQ columns back to rotated order: ``(deq fp32 or None, q int8 or None)``."""
    M, N = q.shape
    dev = q.device
    deq = torch.empty((M, N), dtype=torch.float32, device=dev) if want_deq else None
    qs = torch.empty((M, N), dtype=torch.int8, device=dev) if want_q else None
    L.check(L.load().qi8_ldlq_finish(L.ptr(q), M, N, L.ptr(scale), L.ptr(cols), L.ptr(deq), L.ptr(qs),
                                     L.stream_ptr(dev)), "qi8_ldlq_finish")
    return deq, qs


def device_status(reset: bool = True) -> None:
    """Raise if a kernel's bounded wait expired since the last check."""
    L.check(L.load().qi8_device_status(int(reset)), "device status")
