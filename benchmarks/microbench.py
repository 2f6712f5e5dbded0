"""Kernel micro-benchmarks of the QuIP W8A8 path (one GPU).

    python benchmarks/microbench.py rotate   # K1 rotate+quant, K3 unrotate
    python benchmarks/microbench.py quant    # K1 per-token quant (+ fused GELU)
    python benchmarks/microbench.py gemm     # K2 block-scaled / per-row GEMM
    python benchmarks/microbench.py gemm_stack  # K2 on the Flux / T5 stacks' largest linears
    python benchmarks/microbench.py convert  # K4 QuIP conversion
    python benchmarks/microbench.py ldlq     # default converter: fp64 Hinv factorization, LDLQ pass
    python benchmarks/microbench.py gemm_ksweep  # K2 plain GEMM over K at fixed M, N

Each case is timed with CUDA events around one launch, median of ``--iters``
launches, with a 256 MB buffer rewritten between launches so every launch
reads its inputs from HBM.  Prints one JSON object: case -> [us, GB/s or
TOPS].  ``--profile`` runs every case ``--iters`` times without timing (the
form to run under ncu).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from convert_to_quant_quip_int8_b200 import _lib as L  # noqa: E402
from convert_to_quant_quip_int8_b200 import ops  # noqa: E402


def _timer(flush: torch.Tensor, iters: int, profile: bool):
    def run(fn):
        for _ in range(2):
            fn()
        if profile:
            for _ in range(iters):
                fn()
            torch.cuda.synchronize()
            return float("nan")
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


def _signs(n: int, dev) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(n)
    return (torch.randint(0, 2, (n,), generator=g) * 2 - 1).float().to(dev)


def rotate_cases(run, dev):
    res = {}
    for T, n, npad in [(512, 4096, 4096), (4096, 3072, 4096), (4608, 15360, 16384)]:
        x = torch.randn(T, n, device=dev).to(torch.bfloat16)
        sv = _signs(npad, dev)
        us = run(lambda: ops.rotate_quant_rows(x, sv, npad))
        res[f"k1_rotate_quant_{T}x{n}->{npad}"] = [us, (T * n * 2 + T * npad + T * 4) / us / 1e3]
        y = torch.randn(T, npad, device=dev)
        us = run(lambda: ops.unrotate_rows(y, sv, n, None, torch.bfloat16))
        res[f"k3_unrotate_{T}x{npad}->{n}"] = [us, (T * npad * 4 + T * n * 2) / us / 1e3]
    return res


def quant_cases(run, dev):
    res = {}
    for n, mode, name in [(3072, L.QI8_Q_TOKEN, "token"), (12288, L.QI8_Q_TOKEN, "token"),
                          (12288, L.QI8_Q_TOKEN | L.QI8_Q_GELU, "gelu_token")]:
        x = torch.randn(4096, n, device=dev).to(torch.bfloat16)
        us = run(lambda: ops.quant_rows(x, mode))
        res[f"k1_{name}_4096x{n}"] = [us, 4096 * (n * 3 + 4) / us / 1e3]
    return res


def gemm_cases(run, dev):
    res = {}
    for M, N, K in [(4096, 12288, 3072), (4096, 3072, 12288)]:
        a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=dev)
        b = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=dev)
        sa = torch.rand(M, 1, device=dev) * 0.01
        sbk = torch.rand(N, K // 128, device=dev) * 0.01
        sb = torch.rand(N, 1, device=dev) * 0.01
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        us = run(lambda: ops.gemm_i8(a, b, sa, L.QI8_S_ROW, sbk, L.QI8_S_ROW_KBLOCK, None, torch.bfloat16, out=out))
        res[f"k2_block_{M}x{N}x{K}"] = [us, 2 * M * N * K / us / 1e6]
        us = run(lambda: ops.gemm_i8(a, b, sa, L.QI8_S_ROW, sb, L.QI8_S_ROW, None, torch.bfloat16, out=out))
        res[f"k2_row_{M}x{N}x{K}"] = [us, 2 * M * N * K / us / 1e6]
    # the rotated single linear's GEMM (512 tokens, tensorwise weight scale, fp32 out): the workspace entry
    # (splits K only from K = 8192, so this shape runs one pass) and the plain entry
    M, N, K = 512, 4096, 4096
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=dev)
    b = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=dev)
    sa = torch.rand(M, 1, device=dev) * 0.01
    s1 = torch.full((), 0.003, device=dev)
    out = torch.empty(M, N, dtype=torch.float32, device=dev)
    lib = L.load()
    us = run(lambda: ops.gemm_i8(a, b, sa, L.QI8_S_ROW, s1, L.QI8_S_SCALAR, None, torch.float32, out=out))
    res[f"k2_scalar_splitk_{M}x{N}x{K}"] = [us, 2 * M * N * K / us / 1e6]
    us = run(lambda: L.check(lib.qi8_gemm_i8(L.ptr(a), L.ptr(b), M, N, K, L.ptr(sa), L.QI8_S_ROW, L.ptr(s1),
                                             L.QI8_S_SCALAR, None, 0, L.ptr(out), L.QI8_F32, N, L.QI8_ACT_NONE,
                                             L.stream_ptr(dev))))
    res[f"k2_scalar_onepass_{M}x{N}x{K}"] = [us, 2 * M * N * K / us / 1e6]
    return res


def gemm_stack_cases(run, dev):
    """The stacks' largest GEMMs with per-row weight scales, bias and bf16
    output: Flux single-block linear1 (4608 x 3072 -> 21504) first, then the
    T5-XXL wi projection (4096 x 4096 -> 10240)."""
    res = {}
    for name, M, N, K in [("flux_linear1", 4608, 21504, 3072), ("t5_wi", 4096, 10240, 4096)]:
        a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=dev)
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
        sa = torch.rand(M, 1, device=dev) * 0.01
        sb = torch.rand(N, device=dev) * 0.01
        bias = torch.randn(N, device=dev).to(torch.bfloat16)
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        us = run(lambda: ops.gemm_i8(a, b, sa, L.QI8_S_ROW, sb, L.QI8_S_ROW, bias, torch.bfloat16, out=out))
        res[f"k2_row_{name}_{M}x{N}x{K}"] = [us, 2 * M * N * K / us / 1e6]
    return res


def gemm_tile_cases(run, dev):
    """The comfy block-wise layout's GEMM: per-(token, 128-K block)
    activation scales x 128 x 128 weight-tile scales, bias, fp16 out."""
    res = {}
    M, N, K = 4096, 12288, 3072
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
    sa = torch.rand(M, K // 128, device=dev) * 0.01
    sb = torch.rand(N // 128, K // 128, device=dev) * 0.01
    bias = torch.randn(N, device=dev)
    out = torch.empty(M, N, dtype=torch.float16, device=dev)
    us = run(lambda: ops.gemm_i8(a, b, sa, L.QI8_S_ROW_KBLOCK, sb, L.QI8_S_TILE128, bias, torch.float16, out=out))
    res[f"k2_tile_{M}x{N}x{K}"] = [us, 2 * M * N * K / us / 1e6]
    return res


def convert_cases(run, dev):
    res = {}
    for M, N in [(3072, 3072), (12288, 3072), (3072, 12288)]:
        w = (torch.randn(M, N, device=dev) * 0.02).to(torch.bfloat16)
        Mp, Np = 1 << (M - 1).bit_length(), 1 << (N - 1).bit_length()
        su, sv = _signs(Mp, dev), _signs(Np, dev)
        ws = torch.empty(ops.quip_workspace_bytes(M, N), dtype=torch.uint8, device=dev)
        us = run(lambda: ops.quip_convert(w, su, sv, requant=L.QI8_REQ_BLOCK, want_dequant=False, workspace=ws))
        res[f"k4_quip_convert_block_{M}x{N}"] = [us, M * N * 2 / us / 1e3]
    return res


LDLQ_SIZES = (4096, 16384)


def ldlq_cases(run, dev):
    """qi8_hinv_upper (fp64: Cholesky N^3/3 + triangular inverse N^3/3 flops;
    each launch restores its input first, an N^2 fp64 copy) and qi8_ldlq
    (fp32: M N^2 flops, the input copied back first)."""
    res = {}
    for N in LDLQ_SIZES:
        g = torch.Generator(device=dev).manual_seed(N)
        x = torch.randn(N, N, device=dev, dtype=torch.float64, generator=g)
        h = x @ x.t() / N + torch.eye(N, device=dev, dtype=torch.float64)
        del x
        hrev = torch.tril(h.flip(0).flip(1)).contiguous()
        del h
        h2 = torch.empty_like(hrev)
        holder = {}

        def fact():
            h2.copy_(hrev)
            holder["hinv"] = ops.hinv_upper(h2)[0]
        us = run(fact)
        res[f"hinv_upper_{N}"] = [us, (2.0 / 3.0) * N ** 3 / us / 1e6]
        if "hinv" not in holder:
            fact()
        hinv = holder.pop("hinv")
        del hrev, h2
        M = 4096
        w0 = torch.randn(M, N, device=dev, generator=g) * 0.02
        sc = (w0.abs().amax(1, keepdim=True) / 127).clamp(min=1e-12)
        w = torch.empty_like(w0)

        def pass_():
            w.copy_(w0)
            ops.ldlq(w, hinv, sc)
        us = run(pass_)
        res[f"ldlq_{M}x{N}"] = [us, M * N * N / us / 1e6]
        del w0, w, hinv
        torch.cuda.empty_cache()
    return res


def gemm_ksweep_cases(run, dev):
    """The plain-scale per-row GEMM with bf16 bias and output at fixed M, N
    over K (a per-tile floor shows as time that stops falling with K)."""
    res = {}
    g = torch.Generator(device=dev).manual_seed(0)
    for M, N, K in [(4608, 21504, 1536), (4608, 21504, 3072), (4608, 21504, 6144), (4608, 21504, 12288),
                    (4096, 12288, 3072), (4608, 3072, 15360)]:
        a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-128, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        xs = torch.rand(M, 1, device=dev, generator=g) * 0.01
        ws = torch.rand(N, device=dev, generator=g) * 0.01
        bias = torch.randn(N, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        us = run(lambda: ops.gemm_i8(a, b, xs, L.QI8_S_ROW, ws, L.QI8_S_ROW, bias, torch.bfloat16, out=out))
        res[f"k2_plain_{M}x{N}x{K}"] = [us, 2 * M * N * K / us / 1e6]
        del a, b, out
    return res


CASES = {"rotate": rotate_cases, "quant": quant_cases, "gemm": gemm_cases, "gemm_stack": gemm_stack_cases,
         "gemm_tile": gemm_tile_cases,
         "convert": convert_cases, "ldlq": ldlq_cases, "gemm_ksweep": gemm_ksweep_cases}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--profile", action="store_true")
    ap.add_argument("--small", action="store_true", help="ldlq: only the 4096 size (the form for ncu captures)")
    args = ap.parse_args(argv)
    if args.small:
        global LDLQ_SIZES
        LDLQ_SIZES = (4096,)
    dev = torch.device("cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    res = CASES[args.case](_timer(flush, args.iters, args.profile), dev)
    print(json.dumps({k: [round(v[0], 2), round(v[1], 1)] for k, v in res.items()}))


if __name__ == "__main__":
    main()
