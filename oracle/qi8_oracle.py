"""numpy restatement of the reference's QuIP W8A8 arithmetic (CPU oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  The shipped package
never imports this file; tests, ``smoke()`` and ``bench.py``'s CPU baseline do.

All citations are ``path:line`` inside the reference project
(ThunderFun/convert_to_quant_QuIP_INT8 v0.8.2, package ``convert_to_quant``).

Conventions
-----------
* bf16 values travel as ``uint16`` bit patterns (numpy has no bfloat16);
  :func:`bf16_to_f32` / :func:`f32_to_bf16` convert (round-to-nearest-even).
* Every float32 expression below is evaluated with numpy float32 scalars and
  arrays, which are IEEE-754 single operations with no fused multiply-add, i.e.
  the same rounding the reference's torch CPU kernels perform.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

INT8_SYMMETRIC_MAX = 127  # constants.py INT8_SYMMETRIC_MAX


# --------------------------------------------------------------------------
# bf16 / f16 bit helpers
# --------------------------------------------------------------------------

def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (torch ``.to(bfloat16)``)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    out = rounded.astype(np.uint16)
    if nan.any():
        out = np.where(nan, ((u >> np.uint64(16)) | np.uint64(0x40)).astype(np.uint16), out)
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_to_f32(f32_to_bf16(x))


def next_power_of_two(n: int) -> int:
    """utils/hadamard.py:85-88."""
    if n <= 0:
        return 1
    return 2 ** (n - 1).bit_length()


def is_power_of_two(n: int) -> bool:
    """utils/hadamard.py:81-82."""
    return n > 0 and (n & (n - 1)) == 0


# --------------------------------------------------------------------------
# Fast Walsh-Hadamard transform
# --------------------------------------------------------------------------

def fwht_rows(x: np.ndarray, normalize: bool = True) -> np.ndarray:
    """FWHT along the last axis, fp32.

    Restates ``_fast_hadamard_transform_core_optimized``
    (utils/hadamard.py:114-159): butterfly stages in ascending stride order
    h = 1, 2, 4, ... with ``(a, b) -> (a + b, a - b)`` where ``a`` is the lower
    index, each stage an fp32 add/sub, then (if ``normalize``) one fp32
    multiply by ``float32(1.0 / sqrt(n))`` (hadamard.py:155-157).
    """
    a = np.ascontiguousarray(x, dtype=np.float32)
    shape = a.shape
    n = shape[-1]
    if not is_power_of_two(n):
        raise ValueError(f"Last dimension must be a power of 2, got {n}")
    a = a.reshape(-1, n)
    rows = a.shape[0]
    h = 1
    while h < n:
        v = a.reshape(rows, n // (2 * h), 2, h)
        lo = v[:, :, 0, :]
        hi = v[:, :, 1, :]
        a = np.stack([lo + hi, lo - hi], axis=2).reshape(rows, n)
        h *= 2
    if normalize:
        a = a * np.float32(1.0 / math.sqrt(n))
    return a.reshape(shape)


def fwht_cols(x: np.ndarray, normalize: bool = True) -> np.ndarray:
    """FWHT along axis -2 (the reference's ``fht(W.t()).t()``, quip_int8.py:545, 1490)."""
    return np.ascontiguousarray(np.swapaxes(fwht_rows(np.swapaxes(x, -1, -2), normalize), -1, -2))


def fwht_2d(x: np.ndarray, normalize: bool = True) -> np.ndarray:
    """``fast_hadamard_transform_2d`` (utils/hadamard.py:467-516).

    Last-dim FWHT then row-dim FWHT, both un-normalized, then one fp32
    division by ``float32(sqrt(rows * cols))`` (hadamard.py:512-514).
    """
    r, c = x.shape[-2], x.shape[-1]
    y = fwht_rows(x, normalize=False)
    y = fwht_cols(y, normalize=False)
    if normalize:
        y = y / np.float32(math.sqrt(r * c))
    return y


# --------------------------------------------------------------------------
# Activation / weight quantization
# --------------------------------------------------------------------------

def _rint_clamp_i8(v: np.ndarray, lo: float, hi: float) -> np.ndarray:
    return np.clip(np.rint(v), np.float32(lo), np.float32(hi)).astype(np.int8)


def quantize_int8_axiswise(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Per-row (per-token) absmax int8 quantization, utils/float_utils.py:9-37.

    ``scale = (amax(|x|) / 127.0).clamp(min=1e-30)`` (fp32 division);
    ``q = round_half_even(x * reciprocal(scale)).clamp(-128, 127)`` where
    ``1.0 / scale`` is torch's ``reciprocal(scale) * 1.0`` (float_utils.py:35-36).
    ``x`` is float32 (bf16 inputs are widened exactly first).
    Returns ``(q int8 [..., n], scale float32 [..., 1])``.
    """
    xf = np.asarray(x, dtype=np.float32)
    amax = np.abs(xf).max(axis=-1, keepdims=True).astype(np.float32)
    scale = np.maximum(amax / np.float32(127.0), np.float32(1e-30)).astype(np.float32)
    rcp = (np.float32(1.0) / scale).astype(np.float32)
    q = _rint_clamp_i8(xf * rcp, -128.0, 127.0)
    return q, scale


def quantize_int8_tensorwise(x: np.ndarray) -> Tuple[np.ndarray, np.float32]:
    """Whole-tensor absmax int8 quantization, utils/float_utils.py:40-66."""
    xf = np.asarray(x, dtype=np.float32)
    amax = np.float32(np.abs(xf).max())
    scale = np.float32(max(np.float32(amax / np.float32(127.0)), np.float32(1e-30)))
    rcp = np.float32(np.float32(1.0) / scale)
    q = _rint_clamp_i8(xf * rcp, -128.0, 127.0)
    return q, scale


def _trunc_i8(v: np.ndarray) -> np.ndarray:
    """fp32 -> int8 conversion of the Triton kernels: round toward zero,
    saturating, NaN -> 0 (PTX ``cvt.rzi.s8.f32``)."""
    v = np.where(np.isnan(v), np.float32(0), v)
    return np.clip(np.trunc(v), -128, 127).astype(np.int8)


def act_quant(x: np.ndarray, block_size: int = 128) -> Tuple[np.ndarray, np.ndarray]:
    """Triton ``act_quant`` (comfy/int8_kernels.py:72-123).

    Per (row, 128-block): ``s = amax / 127`` (fp32, no floor), ``y = x / s``
    (fp32 division), converted to int8 by truncation.  Returns
    ``(y int8 [..., K], s float32 [..., K/block])``.
    """
    xf = np.asarray(x, dtype=np.float32)
    K = xf.shape[-1]
    assert K % block_size == 0
    xb = xf.reshape(*xf.shape[:-1], K // block_size, block_size)
    amax = np.abs(xb).max(axis=-1).astype(np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = (xb / s[..., None]).astype(np.float32)
    return _trunc_i8(y).reshape(xf.shape), s


def act_dequant(q: np.ndarray, s: np.ndarray, block_size: int = 128) -> np.ndarray:
    """Triton ``act_dequant`` (comfy/int8_kernels.py:126-179): ``y = q * s`` (fp32)."""
    K = q.shape[-1]
    qb = q.astype(np.float32).reshape(*q.shape[:-1], K // block_size, block_size)
    return (qb * s.astype(np.float32)[..., None]).reshape(q.shape)


def weight_quant(w: np.ndarray, block_size: int = 128) -> Tuple[np.ndarray, np.ndarray]:
    """Triton ``weight_quant`` (comfy/int8_kernels.py:182-253).

    Per 128x128 tile: ``s = max(amax / 127, 1e-8)``, ``y = trunc(x / s)``.
    Returns ``(y int8 [M, N], s float32 [M/bs, N/bs])``.
    """
    wf = np.asarray(w, dtype=np.float32)
    M, N = wf.shape
    t = wf.reshape(M // block_size, block_size, N // block_size, block_size)
    amax = np.abs(t).max(axis=(1, 3)).astype(np.float32)
    s = np.maximum((amax / np.float32(127.0)).astype(np.float32), np.float32(1e-8))
    y = (t / s[:, None, :, None]).astype(np.float32)
    return _trunc_i8(y).reshape(M, N), s


def weight_dequant(q: np.ndarray, s: np.ndarray, block_size: int = 128) -> np.ndarray:
    """Triton ``weight_dequant`` (comfy/int8_kernels.py:256-330): ``y = q * s`` per tile."""
    M, N = q.shape
    t = q.astype(np.float32).reshape(M // block_size, block_size, N // block_size, block_size)
    return (t * s.astype(np.float32)[:, None, :, None]).reshape(M, N)


# --------------------------------------------------------------------------
# GEMM and epilogues
# --------------------------------------------------------------------------

def int_mm(a: np.ndarray, b_nk: np.ndarray) -> np.ndarray:
    """int8 x int8 -> int32, ``C = A @ B^T`` with B stored [N, K].

    Semantics of ``mm_8bit`` (comfy/int8_matmul_kernels.py:82-110) /
    ``torch._int_mm``.  Evaluated as a float64 matmul, which is exact here:
    every partial sum is an integer of magnitude <= 128*128*K < 2**53.
    """
    a64 = np.asarray(a, dtype=np.float64)
    b64 = np.asarray(b_nk, dtype=np.float64)
    return (a64 @ b64.T).astype(np.int64).astype(np.int32)


def linear_w8a8_epilogue(acc: np.ndarray, x_s: np.ndarray, w_s: np.ndarray,
                         bias: Optional[np.ndarray]) -> np.ndarray:
    """Epilogue of ``optimized_linear`` (comfy/quant_ops.py:471-474).

    ``res.float() * (x_s * w_s)`` (fp32, the product of the two scales first),
    ``+= bias`` (fp32), result float32 (the caller rounds to the input dtype).
    ``x_s`` is [T, 1]; ``w_s`` is a scalar (tensorwise) or [N] (axiswise /
    per-row).
    """
    xs = np.asarray(x_s, dtype=np.float32).reshape(-1, 1)
    ws = np.asarray(w_s, dtype=np.float32)
    s = (xs * ws.reshape(1, -1)) if ws.ndim > 0 and ws.size > 1 else (xs * ws.reshape(()))
    y = acc.astype(np.float32) * s.astype(np.float32)
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32).reshape(1, -1)
    return y.astype(np.float32)


def linear_w8a8(x: np.ndarray, w_q: np.ndarray, w_s: np.ndarray,
                bias: Optional[np.ndarray]) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Tensorwise / axiswise W8A8 linear (comfy/quant_ops.py:461-475).

    Returns ``(x_q, x_s, acc_int32, y_f32)``; ``y`` before the final cast.
    """
    x_q, x_s = quantize_int8_axiswise(x)
    acc = int_mm(x_q, w_q)
    return x_q, x_s, acc, linear_w8a8_epilogue(acc, x_s, w_s, bias)


def int8_gemm_block(a: np.ndarray, a_s: np.ndarray, b: np.ndarray, b_s: np.ndarray,
                    bias: Optional[np.ndarray] = None, block_size: int = 128,
                    b_layout: str = "tile") -> np.ndarray:
    """Block-K promoted GEMM of ``int8_gemm`` / ``int8_addmm``
    (comfy/int8_kernels.py:368-404 and 446-494).

    ``acc += float(A_kb @ B_kb^T) * a_s[m, kb] * b_s[n // 128, kb]`` summed in
    kb order (fp32), ``+ bias``; returns float32 (the reference stores fp16).
    ``a_s`` is [M, K/128] or a per-token [M] / [M, 1] scale (applied every kb).
    ``b_layout="row"`` selects the per-output-row layout [N, K/128] written by
    the QuIP block requant (converters/quip_int8.py:1622-1628).
    """
    M, K = a.shape
    N = b.shape[0]
    KB = K // block_size
    a_s = np.asarray(a_s, dtype=np.float32).reshape(M, -1)
    b_s = np.asarray(b_s, dtype=np.float32).reshape(-1, KB)
    acc = np.zeros((M, N), dtype=np.float32)
    a32 = np.asarray(a, dtype=np.float32)
    b32 = np.asarray(b, dtype=np.float32)
    for kb in range(KB):
        sl = slice(kb * block_size, (kb + 1) * block_size)
        # the int32 partial of one K block: every partial sum is an integer of
        # magnitude <= 128*128*block_size <= 2**24, exact in fp32 in any order
        part = a32[:, sl] @ b32[:, sl].T
        sa = a_s[:, kb if a_s.shape[1] > 1 else 0][:, None]
        if b_layout == "row":
            sb = b_s[:, kb][None, :]
        else:
            sb = np.repeat(b_s[:, kb], block_size)[:N][None, :]
        acc = acc + (part * sa).astype(np.float32) * sb
    if bias is not None:
        acc = acc + np.asarray(bias, dtype=np.float32)[None, :]
    return acc.astype(np.float32)


def _block_requant_trunc(y: np.ndarray, out_block_size: int) -> Tuple[np.ndarray, np.ndarray]:
    """Per (row, ``out_block_size`` columns) requantization of the Triton
    fused kernels (comfy/int8_kernels.py:755-767, 1200-1213):
    ``scale = max(amax / 127, 1e-8)``, ``q = int8(clamp(y / scale, -127, 127))``
    (fp32 division, conversion by truncation)."""
    M, N = y.shape
    assert N % out_block_size == 0
    r = np.asarray(y, np.float32).reshape(M, N // out_block_size, out_block_size)
    amax = np.abs(r).max(axis=2).astype(np.float32)
    scale = np.maximum((amax / np.float32(127.0)).astype(np.float32), np.float32(1e-8)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        v = (r / scale[..., None]).astype(np.float32)
    v = np.minimum(np.maximum(v, np.float32(-127.0)), np.float32(127.0))
    return _trunc_i8(v).reshape(M, N), scale


def int8_gemm_quant(a: np.ndarray, a_s: np.ndarray, b: np.ndarray, b_s: np.ndarray,
                    bias: Optional[np.ndarray] = None, out_block_size: int = 128, block_size: int = 128,
                    b_layout: str = "tile") -> Tuple[np.ndarray, np.ndarray]:
    """Fused GEMM + output quantization, ``int8_gemm_quant`` /
    ``int8_addmm_quant`` (comfy/int8_kernels.py:684-797, 800-917, 920-1089):
    the block-promoted fp32 accumulator of :func:`int8_gemm_block`
    (``acc += fp32(A_kb B_kb^T) * a_s * b_s`` in K-block order), ``+ bias``,
    then the per-(row, 128-column block) int8 requantization.  Returns
    ``(q int8 [M, N], scale float32 [M, N / out_block_size])``."""
    acc = int8_gemm_block(a, a_s, b, b_s, bias, block_size, b_layout)
    return _block_requant_trunc(acc, out_block_size)


def _erf_f32(x: np.ndarray) -> np.ndarray:
    """erf of float32 inputs evaluated in double and rounded to float32 (the
    reference's Triton ``tl.math.erf`` as executed: math.erf per element)."""
    xd = np.asarray(x, dtype=np.float64)
    try:
        from scipy.special import erf as _erf
        return _erf(xd).astype(np.float32)
    except ImportError:  # pragma: no cover
        return np.vectorize(math.erf)(xd).astype(np.float32)


def int8_gelu(q: np.ndarray, s: np.ndarray, block_size: int = 128) -> Tuple[np.ndarray, np.ndarray]:
    """Fused int8 GELU, ``int8_gelu_kernel`` (comfy/int8_kernels.py:1122-1213):
    ``v = fp32(q) * s`` per (row, block); ``e = erf(v / fp32(1.41421356237))``;
    ``g = (v * 0.5) * (1 + e)`` (all fp32, left to right); then the same
    per-(row, block) requantization as the fused GEMM.  Returns
    ``(q int8 [M, N], scale float32 [M, N / block_size])``."""
    M, N = q.shape
    v = (q.astype(np.float32).reshape(M, N // block_size, block_size)
         * np.asarray(s, np.float32).reshape(M, N // block_size)[..., None]).astype(np.float32)
    e = _erf_f32((v / np.float32(1.41421356237)).astype(np.float32))
    g = ((v * np.float32(0.5)).astype(np.float32) * (np.float32(1.0) + e).astype(np.float32)).astype(np.float32)
    return _block_requant_trunc(g.reshape(M, N), block_size)


def gptq_quant_block(w: np.ndarray, hinv: np.ndarray, scale) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """GPTQ / LDLQ error-feedback quantization of one column block,
    ``gptq_quant_block_kernel`` (comfy/gptq_kernels.py:11-85), every row in
    parallel.  ``w`` [M, B] fp32 (returned updated, as the kernel updates it in
    place), ``hinv`` [B, B] fp32, ``scale`` a scalar or [M, 1].  For each column
    j in order: ``s = max(|scale|, 1e-12)``, ``q = clamp(rint(w_j / s), -127, 127)``
    (the kernel's floor/fraction test is round-half-even), ``d = max(|hinv[j, j]|,
    1e-12)``, ``err = (w_j - q * s) / d``, then ``w_k -= err * hinv[j, k]`` for
    k > j (fp32, separately rounded).  Returns ``(q int8 [M, B], err fp32 [M, B],
    w fp32 [M, B])``."""
    W = np.array(w, dtype=np.float32, copy=True)
    H = np.asarray(hinv, dtype=np.float32)
    M, B = W.shape
    sc = np.asarray(scale, dtype=np.float32).reshape(-1)
    sc = np.maximum(np.abs(sc if sc.size > 1 else np.full(M, sc[0], np.float32)), np.float32(1e-12))
    Q = np.zeros((M, B), np.int8)
    E = np.zeros((M, B), np.float32)
    for j in range(B):
        wj = W[:, j].copy()
        q = np.clip(np.rint((wj / sc).astype(np.float32)), np.float32(-127.0), np.float32(127.0)).astype(np.float32)
        Q[:, j] = q.astype(np.int8)
        d = np.maximum(np.abs(H[j, j]), np.float32(1e-12)).astype(np.float32)
        err = ((wj - (q * sc).astype(np.float32)).astype(np.float32) / d).astype(np.float32)
        E[:, j] = err
        if j + 1 < B:
            W[:, j + 1:] = (W[:, j + 1:] - (err[:, None] * H[j, j + 1:][None, :]).astype(np.float32)).astype(np.float32)
    return Q, E, W


def gelu_f32(x: np.ndarray) -> np.ndarray:
    """Exact-erf GELU ``0.5 x (1 + erf(x / sqrt 2))`` (torch ``F.gelu`` default)."""
    xf = np.asarray(x, dtype=np.float64)
    try:
        from scipy.special import erf as _erf
        v = _erf(xf / math.sqrt(2.0))
    except ImportError:  # pragma: no cover
        from math import erf
        v = np.vectorize(erf)(xf / math.sqrt(2.0))
    return (0.5 * xf * (1.0 + v)).astype(np.float32)


# --------------------------------------------------------------------------
# Online QuIP activation path (rotated W8A8 linear)
# --------------------------------------------------------------------------

def rotate_rows(x: np.ndarray, sign: Optional[np.ndarray], n_pad: int,
                normalize: bool = True) -> np.ndarray:
    """``FWHT(pad(x).float() * s_v)`` -- steps 1-2 of ``quip_int8_matmul``
    (comfy/int8_kernels.py:1411-1428) with the pad-to-power-of-two rule of
    converters/quip_int8.py:450-451, 539-547 (zero padding on the right)."""
    xf = np.asarray(x, dtype=np.float32)
    T, n = xf.shape
    xp = np.zeros((T, n_pad), dtype=np.float32)
    xp[:, :n] = xf
    if sign is not None:
        xp = xp * np.asarray(sign, dtype=np.float32)[None, :]
    return fwht_rows(xp, normalize)


def rotate_quant_rows(x: np.ndarray, sign: Optional[np.ndarray], n_pad: int) -> Tuple[np.ndarray, np.ndarray]:
    """K1: sign -> FWHT -> per-token absmax int8 (quantize_int8_axiswise)."""
    return quantize_int8_axiswise(rotate_rows(x, sign, n_pad))


def unrotate_rows(y_had: np.ndarray, sign_u: Optional[np.ndarray], n_out: int,
                  bias: Optional[np.ndarray]) -> np.ndarray:
    """K3: ``FWHT(y_had) * s_u`` (comfy/int8_kernels.py:1446-1450), sliced to
    ``n_out`` columns, ``+ bias`` in fp32.  Returns float32 (caller rounds)."""
    y = fwht_rows(np.asarray(y_had, dtype=np.float32), True)
    if sign_u is not None:
        y = y * np.asarray(sign_u, dtype=np.float32)[None, :]
    y = y[:, :n_out]
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)[None, :]
    return np.ascontiguousarray(y, dtype=np.float32)


def quip_linear_w8a8(x: np.ndarray, q_t: np.ndarray, w_s: np.ndarray, s_u: np.ndarray,
                     s_v: np.ndarray, n_out: int, bias: Optional[np.ndarray]):
    """Transformed-space W8A8 linear: K1 -> int32 GEMM -> fp32 scale -> K3.

    ``q_t`` [N_pad, K_pad] int8 with per-row scale ``w_s`` [N_pad] (the
    ``store_transformed`` output of converters/quip_int8.py:1558-1608).
    Returns ``(x_q, x_s, acc, y_had, y)``.
    """
    K_pad = q_t.shape[1]
    x_q, x_s = rotate_quant_rows(x, s_v, K_pad)
    acc = int_mm(x_q, q_t)
    y_had = linear_w8a8_epilogue(acc, x_s, np.asarray(w_s).reshape(-1), None)
    y = unrotate_rows(y_had, s_u, n_out, bias)
    return x_q, x_s, acc, y_had, y


# --------------------------------------------------------------------------
# Offline QuIP weight path (Hadamard incoherence + RTN + requant)
# --------------------------------------------------------------------------

def quip_rotate_weight(w: np.ndarray, s_u: np.ndarray, s_v: np.ndarray) -> np.ndarray:
    """``W' = FHT_N(FHT_M(pad(W) * s_u * s_v^T))``, converters/quip_int8.py:539-551.

    M-direction (columns, via ``.t()``) first, each 1-D transform normalized.
    """
    wf = np.asarray(w, dtype=np.float32)
    M, N = wf.shape
    Mp, Np = s_u.shape[0], s_v.shape[0]
    wp = np.zeros((Mp, Np), dtype=np.float32)
    wp[:M, :N] = wf
    wp = wp * np.asarray(s_u, np.float32)[:, None]
    wp = wp * np.asarray(s_v, np.float32)[None, :]
    wp = fwht_cols(wp, True)
    return fwht_rows(wp, True)


def quip_rtn_rows(wr: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Rotated-space per-row RTN (LDLQ with a diagonal Hinv).

    ``scale = (amax_row / 127).clamp(min=1e-12)`` (converters/quip_int8.py:1272-1274),
    ``Q' = round(W' / scale).clamp(-127, 127)`` (fp32 division, :655-656).
    """
    amax = np.abs(wr).max(axis=1, keepdims=True).astype(np.float32)
    scale = np.maximum(amax / np.float32(INT8_SYMMETRIC_MAX), np.float32(1e-12)).astype(np.float32)
    q = _rint_clamp_i8((wr / scale).astype(np.float32), -127.0, 127.0)
    return q, scale


def quip_unrotate_weight(q: np.ndarray, scale: np.ndarray, s_u: np.ndarray, s_v: np.ndarray,
                         M: int, N: int) -> np.ndarray:
    """Dequant and inverse rotation, converters/quip_int8.py:1452, 1489-1506.

    ``W_dq' = Q' * scale``; ``FHT_N`` (rows) first, then ``FHT_M`` (columns),
    then ``* s_u * s_v``; slice ``[:M, :N]``.
    """
    wd = q.astype(np.float32) * np.asarray(scale, np.float32).reshape(-1, 1)
    wd = fwht_rows(wd, True)
    wd = fwht_cols(wd, True)
    wd = wd * np.asarray(s_u, np.float32)[:, None]
    wd = wd * np.asarray(s_v, np.float32)[None, :]
    return np.ascontiguousarray(wd[:M, :N])


def quip_inverse_rotate(wr: np.ndarray, s_u: np.ndarray, s_v: np.ndarray, M: int, N: int) -> np.ndarray:
    """Inverse incoherence rotation of a rotated-space matrix,
    converters/quip_int8.py:1489-1506: ``FHT_N`` (rows) first, then ``FHT_M``
    (columns), then ``* s_u * s_v``; slice ``[:M, :N]``."""
    wd = fwht_rows(np.asarray(wr, np.float32), True)
    wd = fwht_cols(wd, True)
    wd = wd * np.asarray(s_u, np.float32)[:, None]
    wd = wd * np.asarray(s_v, np.float32)[None, :]
    return np.ascontiguousarray(wd[:M, :N])


def quip_requant(w: np.ndarray, scheme: str = "tensor", per_row: bool = True,
                 block_size: int = 128) -> Tuple[np.ndarray, np.ndarray]:
    """Original-space requantization, converters/quip_int8.py:1614-1669.

    * ``block`` (when ``N % block_size == 0``): scale [M, N/bs, 1] per row x K-block;
    * ``tensor`` with ``per_row``: scale [M, 1]; otherwise a 0-d global scale.
    Scales clamp at 1e-12; ``Q = round(W / scale).clamp(-127, 127)`` (division).
    """
    M, N = w.shape
    if scheme == "block" and N % block_size == 0:
        wr = w.reshape(M, N // block_size, block_size)
        amax = np.abs(wr).max(axis=2, keepdims=True).astype(np.float32)
        scale = np.maximum(amax / np.float32(INT8_SYMMETRIC_MAX), np.float32(1e-12)).astype(np.float32)
        q = _rint_clamp_i8((wr / scale).astype(np.float32), -127.0, 127.0).reshape(M, N)
        return q, scale
    if per_row:
        amax = np.abs(w).max(axis=1, keepdims=True).astype(np.float32)
        scale = np.maximum(amax / np.float32(INT8_SYMMETRIC_MAX), np.float32(1e-12)).astype(np.float32)
    else:
        scale = np.array(max(np.float32(np.float32(np.abs(w).max()) / np.float32(INT8_SYMMETRIC_MAX)),
                             np.float32(1e-12)), dtype=np.float32)
    q = _rint_clamp_i8((w / scale).astype(np.float32), -127.0, 127.0)
    return q, scale


def quip_convert(w: np.ndarray, s_u: np.ndarray, s_v: np.ndarray, requant_scheme: str = "tensor",
                 per_row: bool = True, store_transformed: bool = False, block_size: int = 128):
    """QuIP Hadamard conversion with identity Hessian, no diagonal rescaling,
    no random permutation, no act-order (``QuIPInt8Converter.convert``,
    converters/quip_int8.py:1031-1682): rotate, rotated-space RTN, inverse,
    requant.  Returns ``(q, scale, dequantized_weight)`` -- with
    ``store_transformed`` the padded rotated ``Q'`` and its [M_pad, 1] scale.
    """
    M, N = w.shape
    wr = quip_rotate_weight(w, s_u, s_v)
    qr, sr = quip_rtn_rows(wr)
    deq = quip_unrotate_weight(qr, sr, s_u, s_v, M, N)
    if store_transformed:
        return qr, sr, deq
    q, s = quip_requant(deq, requant_scheme, per_row, block_size)
    return q, s, deq


# --------------------------------------------------------------------------
# QuIP with the reference's defaults: diagonal rescaling, random permutation,
# damping, act-order, fp64 Hessian factorization, blocked lazy LDLQ
# --------------------------------------------------------------------------

def _cascade_rows(rows: np.ndarray) -> np.ndarray:
    """torch's CPU ``multi_row_sum``: a four-level cascade down axis 0, every
    trailing column independent.  Level 0 adds ``step = 2**max(4,
    ceil_log2(size) // 4)`` rows in order, is added into level 1 and cleared;
    level j carries into level j+1 whenever the row count is a multiple of
    ``step**j``; left-over rows go into level 0; finally ``acc0 += acc1;
    acc0 += acc2; acc0 += acc3``."""
    size = rows.shape[0]
    lp = max(4, (int(math.ceil(math.log2(size))) if size > 1 else 0) // 4)
    step, mask = 1 << lp, (1 << lp) - 1
    acc = [np.zeros(rows.shape[1:], np.float32) for _ in range(4)]
    i = 0
    while i + step <= size:
        for _ in range(step):
            acc[0] = (acc[0] + rows[i]).astype(np.float32)
            i += 1
        for j in range(1, 4):
            acc[j] = (acc[j] + acc[j - 1]).astype(np.float32)
            acc[j - 1] = np.zeros_like(acc[0])
            if i & (mask << (j * lp)):
                break
    while i < size:
        acc[0] = (acc[0] + rows[i]).astype(np.float32)
        i += 1
    for j in range(1, 4):
        acc[0] = (acc[0] + acc[j]).astype(np.float32)
    return acc[0]


def _row_sum(cols: np.ndarray) -> np.ndarray:
    """torch's CPU ``row_sum``: the M values of a column viewed as [M/4, 4],
    a cascade (:func:`_cascade_rows`) per lane, the M % 4 left-over values
    added to lane 0 in order, then ``lane0 += lane1; += lane2; += lane3``."""
    M = cols.shape[0]
    si = M // 4
    if si:
        p = _cascade_rows(cols[:si * 4].reshape(si, 4, *cols.shape[1:]))
        lanes = [p[k].copy() for k in range(4)]
    else:
        lanes = [np.zeros(cols.shape[1:], np.float32) for _ in range(4)]
    for i in range(si * 4, M):
        lanes[0] = (lanes[0] + cols[i]).astype(np.float32)
    for k in range(1, 4):
        lanes[0] = (lanes[0] + lanes[k]).astype(np.float32)
    return lanes[0]


COLSUM_VEC = 8  # float lanes of the CPU sum kernel torch selects (AVX2 width)


def col_sumsq(w: np.ndarray) -> np.ndarray:
    """``(W ** 2).sum(dim=0)`` in fp32 with torch's CPU summation order
    (converters/quip_int8.py:266).  With N >= 8 columns the reduction runs in
    groups of 4 x 8 columns, each column a :func:`_cascade_rows` over the
    rows, and the last ``N % 32`` columns by :func:`_row_sum`; with N < 8,
    groups of 4 columns by the cascade and the last ``N % 4`` by
    :func:`_row_sum`.  (The multi-threaded split keeps column chunks at
    multiples of 32, so the grouping does not depend on the thread count.)"""
    sq = (np.asarray(w, np.float32) * np.asarray(w, np.float32)).astype(np.float32)
    N = sq.shape[1]
    nv = (N // (4 * COLSUM_VEC)) * 4 * COLSUM_VEC if N >= COLSUM_VEC else (N // 4) * 4
    out = np.zeros(N, np.float32)
    if nv:
        out[:nv] = _cascade_rows(sq[:, :nv])
    if nv < N:
        out[nv:] = _row_sum(sq[:, nv:])
    return out


def diag_rescale(w: np.ndarray, h: Optional[np.ndarray]):
    """``_apply_diagonal_rescaling`` (converters/quip_int8.py:244-287):
    ``D = clamp(float((max(diag H, 1e-12) / max(colsumsq, 1e-12)) ** 0.25), 0.1, 10)``
    with the ratio and the fourth root in fp64; ``W * D`` per column and
    ``(H * Dinv_j) * Dinv_i`` with ``Dinv = 1 / D`` (fp32).  ``h=None`` is the
    identity Hessian.  Returns ``(W_r, H_r, D)``."""
    w = np.asarray(w, np.float32)
    N = w.shape[1]
    hd = np.ones(N, np.float32) if h is None else np.diag(np.asarray(h, np.float32)).copy()
    wtw = np.maximum(col_sumsq(w), np.float32(1e-12))
    hd = np.maximum(hd, np.float32(1e-12))
    D = np.power(hd.astype(np.float64) / wtw.astype(np.float64), 0.25).astype(np.float32)
    D = np.clip(D, np.float32(0.1), np.float32(10.0)).astype(np.float32)
    wr = (w * D[None, :]).astype(np.float32)
    dinv = (np.float32(1.0) / D).astype(np.float32)
    hm = np.eye(N, dtype=np.float32) if h is None else np.asarray(h, np.float32)
    hr = ((hm * dinv[None, :]).astype(np.float32) * dinv[:, None]).astype(np.float32)
    return wr, hr, D


def ldlq_prepare(wrot: np.ndarray, hrot: np.ndarray, perm: np.ndarray, order: np.ndarray,
                 percdamp: float = 0.01):
    """Random permutation, dead-column handling, damping and act-order
    (converters/quip_int8.py:336-340 with :1105-1146): ``W'[:, perm]``,
    ``H'[perm][:, perm]``; ``dead = diag == 0`` gets ``H_ii = 1`` and a zero
    weight column; ``damp = float32(percdamp) * float32(mean(diag, fp64))`` is
    added to the diagonal; then the act-order permutation ``order`` (the
    reference's ``argsort(diag(H), descending=True)``, computed by the caller
    because its tie order is that of torch's unstable CPU sort).  Returns
    ``(W_p fp32 [M, N], H_p fp64 [N, N], damp)``."""
    W = np.asarray(wrot, np.float32)[:, perm].copy()
    H = np.asarray(hrot, np.float32)[perm][:, perm].copy()
    d = np.diag(H).copy()
    dead = d == 0
    idx = np.nonzero(dead)[0]
    H[idx, idx] = 1.0
    W[:, dead] = 0.0
    damp = np.float32(np.float32(percdamp) * np.float32(np.mean(d.astype(np.float64))))
    r = np.arange(H.shape[0])
    H[r, r] = (H[r, r] + damp).astype(np.float32)
    return W[:, order].copy(), H[order][:, order].astype(np.float64), damp


def damped_order_keys(hrot: np.ndarray, perm: np.ndarray, percdamp: float = 0.01) -> np.ndarray:
    """The damped diagonal the act-order sort ranks (converters/quip_int8.py:1105-1117)."""
    d = np.diag(np.asarray(hrot, np.float32))[perm].copy()
    damp = np.float32(np.float32(percdamp) * np.float32(np.mean(d.astype(np.float64))))
    d = np.where(d == 0, np.float32(1.0), d).astype(np.float32)
    return (d + damp).astype(np.float32)


def ldlq_hinv(hp: np.ndarray) -> np.ndarray:
    """``cholesky(cholesky_inverse(cholesky(H)), upper=True)`` in fp64, cast to
    fp32 (converters/quip_int8.py:1195-1199): the upper Cholesky factor U of
    H^-1 (``H^-1 = U^T U``)."""
    L = np.linalg.cholesky(np.asarray(hp, np.float64))
    Li = np.linalg.inv(L)
    Hi = Li.T @ Li
    return np.linalg.cholesky(Hi).T.astype(np.float32)


def _fma_f32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """``fmaf(a, b, c)`` for fp32 arrays: the product is exact in fp64, the sum
    is rounded to fp64 and then to fp32 (differs from one rounding only when
    the fp64 sum lands exactly on an fp32 midpoint)."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def _dot_update(w: np.ndarray, err: np.ndarray, h: np.ndarray, order: str) -> np.ndarray:
    """``w - err @ h`` (fp32).  ``order="blas"``: numpy's fp32 matmul (the
    reference's torch CPU matmul, converters/quip_int8.py:667, 896-899);
    ``order="seq"``: each dot product accumulated by fmaf in index order from
    zero, then subtracted -- the device kernels' order."""
    if order == "blas":
        return (w - (err @ h).astype(np.float32)).astype(np.float32)
    acc = np.zeros((err.shape[0], h.shape[1]), np.float32)
    for k in range(err.shape[1]):
        acc = _fma_f32(err[:, k:k + 1], h[k:k + 1, :], acc)
    return (w - acc).astype(np.float32)


def ldlq_pass(w: np.ndarray, hinv: np.ndarray, scale: np.ndarray, block: int = 128, batch: int = 16,
              order: str = "blas") -> np.ndarray:
    """One LDLQ pass, ``_single_ldlq_pass`` + ``_quantize_block_lazy``
    (converters/quip_int8.py:813-945, 638-672): for each ``block`` columns, for
    each ``batch`` of 16 columns quantize them together (``q = clamp(rint(w /
    s), -127, 127)``, ``err = (w - q * s) / max(Hinv_jj, 1e-12)``), update the
    rest of the block with ``err @ Hinv[batch, rest]``; after the block update
    every later column with ``Err_block @ Hinv[block, later]``.  Rows are
    independent.  Returns ``Q'`` int8."""
    W = np.array(w, np.float32, copy=True)
    H = np.asarray(hinv, np.float32)
    s = np.asarray(scale, np.float32).reshape(-1, 1)
    M, N = W.shape
    Q = np.zeros((M, N), np.int8)
    for i1 in range(0, N, block):
        i2 = min(i1 + block, N)
        E = np.zeros((M, i2 - i1), np.float32)
        for j in range(i1, i2, batch):
            e = min(j + batch, i2)
            wb = W[:, j:e]
            q = np.clip(np.rint((wb / s).astype(np.float32)), -127.0, 127.0).astype(np.float32)
            Q[:, j:e] = q.astype(np.int8)
            d = np.maximum(np.diag(H[j:e, j:e]), np.float32(1e-12)).astype(np.float32)
            err = ((wb - (q * s).astype(np.float32)).astype(np.float32) / d[None, :]).astype(np.float32)
            E[:, j - i1:e - i1] = err
            if e < i2:
                W[:, e:i2] = _dot_update(W[:, e:i2], err, H[j:e, e:i2], order)
        if i2 < N:
            W[:, i2:] = _dot_update(W[:, i2:], E, H[i1:i2, i2:], order)
    return Q


def quip_ldlq_scale(wp: np.ndarray) -> np.ndarray:
    """``(amax_row / 127).clamp(min=1e-12)`` on the prepared W (converters/quip_int8.py:1272-1274)."""
    return quip_rtn_rows(wp)[1]


def quip_ldlq_finish(qp: np.ndarray, scale: np.ndarray, cols: np.ndarray, s_u: np.ndarray, s_v: np.ndarray,
                     M: int, N: int, D: Optional[np.ndarray]):
    """Undo act-order and the random permutation (``cols[j]`` is the rotated
    column held at LDLQ position j), dequantize ``Q' * scale``, inverse
    rotation, slice and ``W / D`` (converters/quip_int8.py:1348-1365, 1452,
    1467-1513).  Returns ``(Q' in rotated column order, dequantized W)``."""
    qo = np.zeros_like(qp)
    qo[:, cols] = qp
    deq = quip_unrotate_weight(qo, scale, s_u, s_v, M, N)
    if D is not None:
        deq = (deq / np.maximum(np.asarray(D, np.float32), np.float32(1e-12))[None, :]).astype(np.float32)
    return qo, deq


def lpt_partition(costs, n_parts: int):
    """Longest-processing-time-first assignment of units to ``n_parts`` bins.

    Reference-independent helper for the sharded conversion sweep; returns a
    list of index lists.  Ties are broken by unit index so every rank computes
    the same plan.
    """
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    loads = [0] * n_parts
    parts = [[] for _ in range(n_parts)]
    for i in order:
        j = min(range(n_parts), key=lambda p: (loads[p], p))
        parts[j].append(i)
        loads[j] += costs[i]
    return [sorted(p) for p in parts]
