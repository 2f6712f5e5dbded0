"""The reference's own GPU kernels beside libqi8 on the same B200 (one GPU).

Imports the unmodified reference (``convert_to_quant`` 0.8.2 installed under
``baseline/_ref``) and times, with CUDA events after warm-up (median of
``--iters`` launches, a 256 MB buffer rewritten between launches so inputs
come from HBM):

* ``mm_8bit`` (comfy/int8_matmul_kernels.py:82, Triton, int32 out) vs
  ``qi8_gemm_i8`` int32 out vs ``torch._int_mm`` (cuBLAS) on the Flux / DiT
  GEMM shapes;
* the reference's W8A8 layer path ``optimized_linear`` arithmetic on the GPU
  (its ``quantize_int8_axiswise`` + ``mm_8bit`` + fp32 epilogue, with its
  per-call ``w.t().contiguous()``) vs K1 + K2 (``F.linear`` on a
  ``QuantizedTensor`` here);
* ``int8_addmm`` (comfy/int8_kernels.py:557, block-scaled, fp16 out) vs the
  block-scaled K2;
* ``triton_hadamard_transform`` + ``quantize_int8_axiswise`` (the reference's
  rotated-activation steps, comfy/int8_kernels.py:1424-1428 and
  comfy/quant_ops.py:469) vs K1 ``qi8_rotate_quant_rows``;
* ``act_quant`` (comfy/int8_kernels.py:96) vs ``qi8_quant_rows`` block mode;
* ``QuIPInt8Converter(device="cuda", seed)`` with its defaults
  (converters/quip_int8.py:1031-1669: rescaling, permutation, act-order,
  LDLQ; its own device placement and bf16 autocast) vs this package's
  converter, wall clock per tensor (1 warm-up, median of 3), with the
  fraction of int8 codes the two agree on.

Prints one JSON object: case -> {"ref_us", "qi8_us", "cublas_us"?, "speedup"}.

    python benchmarks/reference_gpu.py [--iters 20]
"""

from __future__ import annotations

import argparse
import json
import logging
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))

from convert_to_quant_quip_int8_b200 import _lib as L  # noqa: E402
from convert_to_quant_quip_int8_b200 import ops  # noqa: E402


def timer(flush, iters):
    def run(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(iters):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        ts.sort()
        return ts[len(ts) // 2]
    return run


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    logging.disable(logging.WARNING)
    from convert_to_quant.comfy import int8_kernels as RK
    from convert_to_quant.comfy.int8_matmul_kernels import mm_8bit
    from convert_to_quant.comfy.hadamard_kernels import triton_hadamard_transform
    from convert_to_quant.utils.float_utils import quantize_int8_axiswise
    logging.disable(logging.NOTSET)
    dev = torch.device("cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    run = timer(flush, args.iters)
    res = {}

    def put(name, ref_us, qi8_us, **extra):
        res[name] = {"ref_us": round(ref_us, 2), "qi8_us": round(qi8_us, 2), "speedup": round(ref_us / qi8_us, 2),
                     **{k: round(v, 2) for k, v in extra.items()}}

    g = torch.Generator(device=dev).manual_seed(0)
    for name, M, N, K in [("flux_linear1", 4608, 21504, 3072), ("flux_linear2", 4608, 3072, 15360),
                          ("dit_w1", 4096, 12288, 3072), ("quip_linear", 512, 4096, 4096)]:
        a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        bt = b.t()  # [K, N] view, as the reference's layer passes w.t()
        bt_c = bt.contiguous()
        ref = run(lambda: mm_8bit(a, bt_c))
        ours = run(lambda: ops.gemm_i8(a, b, out_dtype=torch.int32))
        cub = run(lambda: torch._int_mm(a, bt_c))
        ops_ = 2 * M * N * K
        put(f"int32_gemm_{name}_{M}x{N}x{K}", ref, ours, cublas_us=cub, qi8_tops=ops_ / ours / 1e6,
            ref_tops=ops_ / ref / 1e6, cublas_tops=ops_ / cub / 1e6)
        # the layer: bf16 x -> per-token int8 -> GEMM -> epilogue -> bf16
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        w_s = torch.rand(N, device=dev, generator=g) * 1e-3
        bias = torch.randn(N, device=dev, generator=g).to(torch.bfloat16)

        def ref_layer():
            x_q, x_s = quantize_int8_axiswise(x)
            r = mm_8bit(x_q, b.t().contiguous())
            y = r.float() * (x_s * w_s.unsqueeze(0))
            y += bias
            return y.to(torch.bfloat16)

        def our_layer():
            xq, xs = ops.quant_rows(x, L.QI8_Q_TOKEN)
            return ops.gemm_i8(xq, b, xs, L.QI8_S_ROW, w_s, L.QI8_S_ROW, bias, torch.bfloat16)

        put(f"w8a8_layer_{name}", run(ref_layer), run(our_layer))

    # block-scaled addmm, fp16 out (the reference's BlockWise linear)
    M, N, K = 4096, 12288, 3072
    x = torch.randn(M, K, device=dev, generator=g)
    aq, a_s = RK.act_quant(x)
    bq, b_s = RK.weight_quant(torch.randn(N, K, device=dev, generator=g) * 0.02)
    bias = torch.randn(N, device=dev, generator=g)
    ref = run(lambda: RK.int8_addmm(aq, a_s, bq, b_s, bias))
    ours = run(lambda: ops.gemm_i8(aq, bq, a_s, L.QI8_S_ROW_KBLOCK, b_s, L.QI8_S_TILE128, bias, torch.float16))
    put(f"block_addmm_{M}x{N}x{K}", ref, ours, qi8_tops=2 * M * N * K / ours / 1e6, ref_tops=2 * M * N * K / ref / 1e6)
    ref = run(lambda: RK.act_quant(x))
    ours = run(lambda: ops.quant_rows(x, L.QI8_Q_BLOCK))
    put(f"act_quant_{M}x{K}", ref, ours)

    # rotated activations: signs + FHT + per-token int8
    for T, n in [(512, 4096), (4096, 4096), (4608, 16384)]:
        xr = torch.randn(T, n, device=dev, generator=g).to(torch.bfloat16)
        sv = (torch.randint(0, 2, (n,), device=dev, generator=g) * 2 - 1).float()

        def ref_rot():
            xs = xr.float() * sv.unsqueeze(0)
            return quantize_int8_axiswise(triton_hadamard_transform(xs))

        ours = run(lambda: ops.rotate_quant_rows(xr, sv, n))
        bytes_ = T * n * 3 + T * 4
        put(f"rotate_quant_{T}x{n}", run(ref_rot), ours, qi8_gbs=bytes_ / ours / 1e3)
    # the default QuIP converter, whole tensor (host syncs inside both)
    import time
    from convert_to_quant.converters.quip_int8 import QuIPInt8Converter as RefConv
    from convert_to_quant_quip_int8_b200.converters.quip_int8 import QuIPInt8Converter as Conv

    def wall(fn):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            out = fn()
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t0)
        return sorted(ts)[1] * 1e6, out

    for M, N in [(3072, 3072), (12288, 3072), (3072, 12288)]:
        w = (torch.randn(M, N, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        logging.disable(logging.WARNING)
        ref_us, ref_out = wall(lambda: RefConv(device="cuda", seed=1).convert(w.clone()))
        logging.disable(logging.NOTSET)
        our_us, our_out = wall(lambda: Conv(seed=1).convert(w))
        agree = (ref_out[0].to(dev) == our_out[0]).float().mean().item()
        put(f"quip_convert_defaults_{M}x{N}", ref_us, our_us, q_agreement=agree * 100)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
