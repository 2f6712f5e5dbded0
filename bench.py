"""Benchmark of the QuIP W8A8 quantized-linear path on B200.

Default workload (one step = one forward of the Flux-shaped linear stack):
228 QuIP W8A8 linears (19 double blocks x {img 4096, txt 512 tokens} x
{qkv, proj, mlp0, mlp2} + 38 single blocks x 4608 tokens x {linear1,
linear2}), each = per-token int8 quantization of the bf16 input (K1) + the
tcgen05 int8 GEMM with the fused ``acc * (x_s * w_s) + bias`` epilogue (K2),
per-row ``[N, 1]`` weight scales, captured once as a CUDA graph.
Metric: DiT linear-stack tokens/s (4608 tokens per forward), whole job.

    python bench.py [--gpus N --steps K --warmup W]            # this framework
    python bench.py --impl reference [...]                       # the reference's CPU path
    python bench.py --workload {t5_stack,dit_mlp,quip_linear,conversion}

Multi-GPU (torchrun, one rank per GPU, NCCL for the barrier and the
max-over-ranks timing only): every rank holds all weights and runs every
linear on its 1/N of the tokens (strong scaling, no exchange inside the
linear stack).  ``--shard columns`` column-shards every linear with the
output gather fused into the GEMM epilogue; ``--shard replica`` runs one
whole forward per rank (weak scaling).

The reference arm and the ``cpu_baseline`` leg run the unmodified reference
(``convert_to_quant`` 0.8.2, installed under ``baseline/_ref``) on the host
cores: its ``quantize_int8_axiswise`` (utils/float_utils.py:9-37) and the
arithmetic of its ``optimized_linear`` (comfy/quant_ops.py:461-475) with
``torch._int_mm`` standing in for the Triton ``mm_8bit``, which needs CUDA.
The reference's public ``F.linear(x, QuantizedTensor)`` is not used there: on
CPU it dequantizes the weight (comfy/quant_ops.py:160-170) and, for the
per-row and axis-wise fp32 scales of these stacks, the dequantized weight is
fp32 while the input is bf16, so the fallback matmul raises a dtype error.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from collections import OrderedDict

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
REF_DIR = os.path.join(ROOT, "baseline", "_ref")

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the
# dominant kernel of each workload, from one ncu capture of that launch:
#   ncu --clock-control none --metrics dram__bytes_read.sum,dram__bytes_write.sum \
#       -k regex:gemm_pair_kernel -c 1 python benchmarks/microbench.py gemm_stack --profile --iters 1
# (flux: the single-block linear1 GEMM, 4608 x 3072 -> 21504, per-row scales; t5: with -s 3, the
# wi GEMM, 4096 x 4096 -> 10240).
PROFILED_TRAFFIC = {
    "flux": 81274624 + 145703424,  # read + write; 80 MB of operands, 198 MB of bf16 output (part stays in L2)
    "t5": 59306496 + 35874816,  # one wi GEMM launch, 4096 x 4096 -> 10240 (operands 58.7 MB, output 84 MB)
    # mean of the W1 and W2 block GEMM launches of the DiT pair (ncu --set full capture of both)
    "dit_mlp": 128480000,
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="qi8", choices=["qi8", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="flux_stack",
                    choices=["flux_stack", "t5_stack", "dit_mlp", "quip_linear", "conversion", "conversion_ldlq"],
                    help="flux_stack (default): the 228-linear Flux-shaped stack; t5_stack: the 168-linear T5-XXL "
                         "encoder stack (axis-wise scales); dit_mlp: the DiT MLP pair with block-128 K scales; "
                         "quip_linear: one rotated W8A8 linear (K1 rotate -> K2 -> K3); conversion: the 304-tensor "
                         "QuIP conversion sweep; conversion_ldlq: one Flux double + single block through the "
                         "converter with the reference's defaults (rescaling, permutation, act-order, LDLQ)")
    ap.add_argument("--shard", default="auto", choices=["auto", "replica", "columns", "tokens"],
                    help="stacks on N>1 GPUs: tokens (auto) = full weights, each rank 1/N of the tokens; columns = "
                         "every linear column-sharded with its output gathered on every rank; replica = one batch "
                         "per rank (weak scaling)")
    ap.add_argument("--chunks", type=int, default=4, help="token chunks per column-sharded linear (nccl gather)")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="column-sharded output gather: peer = fused into the GEMM epilogue (stores into every "
                         "rank's IPC-mapped buffer + peer barrier); nccl = chunked NCCL all-gather + re-layout")
    return ap.parse_args()


# ----------------------------------------------------------------- peaks
def measured_peaks():
    """(peaks, kind): the driver-measured copy bandwidth and cuBLAS bf16 burst
    of this pool's B200s, else the earlier measurement on this pool."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def int8_peak():
    """Dense int8 tensor peak = 2 x the bf16 burst figure (B200 runs int8 MMAs
    at twice the bf16 rate); returns (TOPS, note)."""
    p, kind = measured_peaks()
    bf16 = float(p.get("bf16_tflops", 1590.0))
    return 2.0 * bf16, f"dense int8 = 2 x {kind} cuBLAS bf16 burst ({bf16} TF/s)"


def hbm_peak():
    p, kind = measured_peaks()
    return float(p.get("hbm_gbs", 6650.0)), f"{kind} STREAM-style copy bandwidth"


# ------------------------------------------------------------ clock probe
class ClockProbe:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        self.idx = device_index

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), parts[4:8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower().startswith("active")})
        sm = [r[0] for r in rows]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------- distributed
def dist_init():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v: float, world: int, device) -> float:
    if world <= 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def finish(world):
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def timed_region(step, steps, world, device):
    """Runs ``steps`` calls of ``step`` between barriers and device syncs;
    returns the max over ranks of the CUDA-event time (ms) and the clocks."""
    stream = torch.cuda.current_stream(device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockProbe(device.index if device.index is not None else 0) as probe:
        barrier(world)
        torch.cuda.synchronize(device)
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize(device)
        barrier(world)
    return max_over_ranks(t0.elapsed_time(t1), world, device), probe.summary()


def event_time(fn, reps, device):
    """Mean CUDA-event time (ms) of ``fn`` over ``reps`` back-to-back calls on
    the current stream."""
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize(device)
    return a.elapsed_time(b) / reps


# =============================================================== CPU arm
def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_threads() -> int:
    """Give torch every host core (torchrun sets OMP_NUM_THREADS=1); returns the
    thread count torch reports afterwards."""
    torch.set_num_threads(cpu_cores())
    return torch.get_num_threads()


def reference_package():
    """The unmodified reference package from ``baseline/_ref``, or None."""
    if not os.path.isdir(os.path.join(REF_DIR, "convert_to_quant")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import logging
    logging.disable(logging.WARNING)
    try:
        import convert_to_quant.utils.float_utils as fu
        import convert_to_quant.utils.hadamard as had
        import convert_to_quant.comfy.quant_ops as qo
        from convert_to_quant.converters.quip_int8 import QuIPInt8Converter
    except Exception:
        return None
    finally:
        logging.disable(logging.NOTSET)
    return {"fu": fu, "had": had, "qo": qo, "QuIPInt8Converter": QuIPInt8Converter}


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def ref_linear(R, x, w_q, w_s, bias):
    """The reference's W8A8 linear (optimized_linear, comfy/quant_ops.py:461-475)
    on CPU tensors: its quantize_int8_axiswise, the per-call weight transpose,
    torch._int_mm for mm_8bit, the fp32 scale epilogue and the cast back."""
    x_q, x_s = R["fu"].quantize_int8_axiswise(x.reshape(-1, x.shape[-1]))
    res = torch._int_mm(x_q, w_q.t().contiguous())
    res_scaled = res.float() * (x_s * w_s.unsqueeze(0))
    if bias is not None:
        res_scaled += bias
    return res_scaled.to(x.dtype)


class StackCPU:
    """A forward of a linear stack through the reference's CPU path, timed one
    distinct linear shape at a time at its full token count; the forward time
    is the sum over all of the stack's linears of their shape's time."""

    def __init__(self, name: str):
        from convert_to_quant_quip_int8_b200.stack import STACKS
        self.cfg = STACKS[name]
        specs = self.cfg["specs"]()
        self.counts = OrderedDict()
        for s in specs:
            key = (s.tokens, s.k, s.n, s.gelu)
            self.counts[key] = self.counts.get(key, 0) + 1
        self.R = reference_package()
        self.kind = "reference" if self.R is not None else "port"
        self.cases = {}
        for i, key in enumerate(self.counts):
            t, k, n, gelu = key
            x = torch.randn(t, k, generator=_gen(700 + i)).to(torch.bfloat16)
            w = (torch.randn(n, k, generator=_gen(800 + i)) * 0.02).to(torch.bfloat16)
            b = (torch.randn(n, generator=_gen(900 + i)) * 0.01).to(torch.bfloat16) if self.cfg["bias"] else None
            if self.R is not None:
                wq, ws = self.R["fu"].quantize_int8_axiswise(w)
                self.cases[key] = (x, wq, ws.reshape(-1), b, gelu)
            else:
                import oracle as O
                wq, ws = O.quantize_int8_axiswise(w.float().numpy())
                self.cases[key] = (x.float().numpy(), wq, ws.reshape(-1), None if b is None else b.float().numpy(),
                                   gelu)
        self.times = {k: [] for k in self.counts}

    def run(self, key):
        x, wq, ws, b, gelu = self.cases[key]
        t0 = time.perf_counter()
        if self.R is not None:
            xin = torch.nn.functional.gelu(x) if gelu else x
            ref_linear(self.R, xin, wq, ws, b)
        else:
            import oracle as O
            xin = O.round_bf16(O.gelu_f32(x)) if gelu else x
            O.f32_to_bf16(O.linear_w8a8(xin, wq, ws, b)[3])
        self.times[key].append(time.perf_counter() - t0)

    def forward_seconds(self) -> float:
        return sum(c * statistics.median(self.times[k]) for k, c in self.counts.items())

    def sample(self) -> str:
        what = ("the reference's quantize_int8_axiswise + torch._int_mm + optimized_linear epilogue"
                if self.R is not None else "the numpy oracle port (reference package not installed)")
        return (f"one linear of each of the {len(self.counts)} distinct (tokens, in, out) shapes of the stack at its "
                f"full token count through {what}; forward time = sum over the stack's "
                f"{sum(self.counts.values())} linears of their shape's median time")


def cpu_stack_baseline(name: str, passes: int = 1):
    """(tokens/s, seconds per forward, threads, kind, sample) of the reference's
    CPU path on the stack; ``passes`` timed passes over the distinct shapes."""
    threads = cpu_threads()
    st = StackCPU(name)
    first = next(iter(st.counts))
    st.run(first)          # warm the thread pool and allocator
    st.times[first].clear()
    for _ in range(max(1, passes)):
        for key in st.counts:
            st.run(key)
    fwd = st.forward_seconds()
    return st.cfg["tokens"] / fwd, fwd, threads, st.kind, st.sample()


class DitCPU:
    """The DiT MLP pair through the reference's block-wise CPU path: weights in
    its own 128 x 128-tile block format (BlockWiseINT8Layout._weight_quantize_pytorch),
    activations by its block-128 quantizer and the CPU branch of
    _int8_gemm_triton_or_fallback (comfy/quant_ops.py:358-371: dequantize both
    operands, fp32 F.linear), exact-erf GELU between the projections."""

    def __init__(self, tokens: int = 4096):
        from convert_to_quant_quip_int8_b200.workloads import DitMlpPair
        wl = DitMlpPair()
        self.R = reference_package()
        self.kind = "reference" if self.R is not None else "port"
        self.x = wl.activations()[:tokens]
        self.tokens = tokens
        self.ops = wl.ops_per_step(tokens)
        if self.R is not None:
            B = self.R["qo"].BlockWiseINT8Layout
            self.w1 = B._weight_quantize_pytorch(wl.w1(), 128)
            self.w2 = B._weight_quantize_pytorch(wl.w2(), 128)
        else:
            import oracle as O
            self.w1 = O.quip_requant(wl.w1().float().numpy(), "block", True)
            self.w2 = O.quip_requant(wl.w2().float().numpy(), "block", True)

    def step(self):
        if self.R is not None:
            qo = self.R["qo"]
            B = qo.BlockWiseINT8Layout
            aq, a_s = B._activation_quantize_pytorch(self.x, 128)
            h = qo._int8_gemm_triton_or_fallback(aq, a_s, self.w1[0], self.w1[1], 128).to(torch.bfloat16)
            h = torch.nn.functional.gelu(h)
            hq, h_s = B._activation_quantize_pytorch(h, 128)
            return qo._int8_gemm_triton_or_fallback(hq, h_s, self.w2[0], self.w2[1], 128).to(torch.bfloat16)
        import oracle as O
        x = self.x.float().numpy()
        (q1, s1), (q2, s2) = self.w1, self.w2
        xq, xs = O.quantize_int8_axiswise(x)
        h = O.int8_gemm_block(xq, xs, q1, s1.reshape(q1.shape[0], -1), None, b_layout="row")
        h = O.round_bf16(O.gelu_f32(O.round_bf16(h)))
        hq, hs = O.quantize_int8_axiswise(h)
        return O.f32_to_bf16(O.int8_gemm_block(hq, hs, q2, s2.reshape(q2.shape[0], -1), None, b_layout="row"))

    def sample(self):
        return (f"{self.tokens} tokens through both linears via the reference's block-wise CPU path "
                "(act block quant, dequantize both operands, fp32 F.linear, GELU)" if self.R is not None else
                f"{self.tokens} tokens through the numpy oracle port (reference package not installed)")


class QuipLinearCPU:
    """Config 1 through the reference's own rotated forward (quip_int8_matmul,
    comfy/int8_kernels.py:1374-1450) on CPU: signs, its fast_hadamard_transform
    (utils/hadamard.py CPU core), fp32 GEMM against the dequantized
    transformed weight (the Triton quip_matmul_kernel's arithmetic), output
    transform, signs, bias."""

    def __init__(self):
        from convert_to_quant_quip_int8_b200.workloads import SingleQuipLinear
        import oracle as O
        wl = SingleQuipLinear()
        self.R = reference_package()
        self.kind = "reference" if self.R is not None else "port"
        su, sv = wl.signs()
        q, s, _ = O.quip_convert(wl.weight().float().numpy(), su.numpy(), sv.numpy(), store_transformed=True)
        self.q, self.s = torch.from_numpy(q), torch.from_numpy(np.asarray(s).reshape(-1))
        self.su, self.sv = su, sv
        self.x, self.b = wl.activations(), wl.bias()
        self.np_ = (q, np.asarray(s).reshape(-1), su.numpy(), sv.numpy())
        self.ops = 2 * wl.tokens * wl.dim * wl.dim
        self.dim = wl.dim

    def step(self):
        if self.R is not None:
            fht = self.R["had"].fast_hadamard_transform
            x = self.x.float() * self.sv.unsqueeze(0)
            x_had = fht(x)
            y_had = x_had @ (self.q.float() * self.s.unsqueeze(1)).t()
            return (fht(y_had) * self.su.unsqueeze(0) + self.b.float()).to(torch.bfloat16)
        import oracle as O
        q, s, su, sv = self.np_
        return O.quip_linear_w8a8(self.x.float().numpy(), q, s, su, sv, self.dim, self.b.float().numpy())[4]

    def sample(self):
        return ("512 x 4096 -> 4096 through the reference's quip_int8_matmul steps on CPU (its FHT, fp32 GEMM on "
                "the dequantized transformed weight)" if self.R is not None else
                "512 x 4096 -> 4096 through the numpy oracle port (reference package not installed)")


class ConversionCPU:
    """One 3072 x 3072 tensor (padded 4096 x 4096) through the reference's
    QuIPInt8Converter on CPU with the Hadamard/RTN options this build
    implements (per-row tensorwise requant), plus the block-128 requant of
    converters/quip_int8.py:1622-1628 on its dequantized output; the sweep
    time is scaled from it by padded element count."""

    def __init__(self):
        from convert_to_quant_quip_int8_b200.workloads import conversion_sweep_tensors
        self.R = reference_package()
        self.kind = "reference" if self.R is not None else "port"
        self.w = (torch.randn(3072, 3072, generator=_gen(0)) * 0.02).to(torch.bfloat16)
        shapes = [(m, n) for _, m, n in conversion_sweep_tensors()]
        pad = lambda m, n: (1 << (m - 1).bit_length()) * (1 << (n - 1).bit_length())
        self.scale = sum(pad(m, n) for m, n in shapes) / pad(3072, 3072)
        self.n_tensors = len(shapes)

    def step(self):
        if self.R is not None:
            conv = self.R["QuIPInt8Converter"](device="cpu", seed=1000, actorder=False,
                                               use_diagonal_rescaling=False, use_random_permutation=False)
            res = conv.convert(self.w.clone())
            deq = res[2].reshape(3072, 24, 128)
            bs = (deq.abs().amax(dim=2, keepdim=True) / 127).clamp(min=1e-12)
            torch.round(deq / bs).clamp(-127, 127).to(torch.int8)
            return res
        import oracle as O
        from convert_to_quant_quip_int8_b200.workloads import quip_signs
        su, sv = (t.numpy() for t in quip_signs(1000, 4096, 4096))
        q, s, deq = O.quip_convert(self.w.float().numpy(), su, sv, "tensor")
        return O.quip_requant(deq, "block")

    def sample(self):
        return ("one 3072 x 3072 tensor through the reference's QuIPInt8Converter (Hadamard/RTN options, per-row "
                "requant) + block-128 requant, scaled to the 304-tensor sweep by padded element count"
                if self.R is not None else "one 3072 x 3072 tensor through the numpy oracle converter, scaled")


def ldlq_cost(m: int, n: int) -> float:
    """Relative cost of the default QuIP conversion of an [m, n] weight:
    the reference's fp64 chol + cholesky_inverse + chol (4/3 N^3) plus the
    LDLQ pass (M N^2), at the padded sizes."""
    mp, np_ = 1 << (m - 1).bit_length(), 1 << (n - 1).bit_length()
    return 4.0 / 3.0 * np_ ** 3 + mp * np_ ** 2


class LdlqCPU:
    """CPU baseline of the default converter: the reference's
    QuIPInt8Converter with its defaults (diagonal rescaling, random
    permutation, act-order, damping, fp64 factorization, LDLQ, per-row
    requant) on one 3072 x 3072 tensor, scaled to the 10-tensor block set by
    :func:`ldlq_cost`.  (At N_pad >= 8192 the reference's CPU-only run takes
    its checkpointed LDLQ branch, so the larger tensors are not sampled.)"""

    def __init__(self):
        from convert_to_quant_quip_int8_b200.workloads import ldlq_block_tensors
        self.R = reference_package()
        self.kind = "reference" if self.R is not None else "port"
        self.w = (torch.randn(3072, 3072, generator=_gen(0)) * 0.02).to(torch.bfloat16)
        shapes = [(m, n) for _, m, n in ldlq_block_tensors()]
        self.scale = sum(ldlq_cost(m, n) for m, n in shapes) / ldlq_cost(3072, 3072)
        self.n_tensors = len(shapes)

    def step(self):
        if self.R is not None:
            return self.R["QuIPInt8Converter"](device="cpu", seed=1000).convert(self.w.clone())
        import oracle as O
        from convert_to_quant_quip_int8_b200.workloads import quip_signs
        w = self.w.float().numpy()
        wr, hr, D = O.diag_rescale(w, None)
        su, sv = (t.numpy() for t in quip_signs(1000, 4096, 4096))
        wrot = O.quip_rotate_weight(wr, su, sv)
        hpad = np.zeros((4096, 4096), np.float32)
        hpad[:3072, :3072] = hr
        hrot = O.quip_rotate_weight(hpad, sv, sv)
        perm = np.random.default_rng(1000).permutation(4096)
        order = np.argsort(-O.damped_order_keys(hrot, perm), kind="stable")
        wp, hp, _ = O.ldlq_prepare(wrot, hrot, perm, order)
        q = O.ldlq_pass(wp, O.ldlq_hinv(hp), O.quip_ldlq_scale(wp))
        return q

    def sample(self):
        return ("one 3072 x 3072 tensor through the reference's QuIPInt8Converter with its defaults, scaled to "
                "the 10-tensor block set by 4/3 N^3 + M N^2 at the padded sizes" if self.R is not None else
                "one 3072 x 3072 tensor through the numpy oracle's default-converter steps, scaled")


def cpu_timed(step, steps, warmup):
    for _ in range(max(0, warmup)):
        step()
    ts = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def cpu_point(workload: str, steps: int = 1, warmup: int = 1):
    """The CPU baseline of a non-stack workload: (value, unit, seconds per
    step, threads, kind, sample)."""
    threads = cpu_threads()
    if workload == "dit_mlp":
        c = DitCPU()
        med = cpu_timed(c.step, steps, warmup)
        return c.ops / med / 1e12, "TOPS", med, threads, c.kind, c.sample()
    if workload == "quip_linear":
        c = QuipLinearCPU()
        med = cpu_timed(c.step, steps, warmup)
        return c.ops / med / 1e12, "TOPS", med, threads, c.kind, c.sample()
    c = LdlqCPU() if workload == "conversion_ldlq" else ConversionCPU()
    med = cpu_timed(c.step, steps, warmup)
    return c.n_tensors / (med * c.scale), "tensors/s", med * c.scale, threads, c.kind, c.sample()


def cpu_baseline_field(value, unit, threads, kind, sample, seconds):
    return {"value": round(value, 4), "unit": unit, "cores": threads, "kind": kind, "sample": sample,
            "seconds_per_step": round(seconds, 3)}


# ============================================================ GPU arms
def main_stack(args):
    """Configs 3 and 4: a whole linear stack per step (K1 + K2 per linear),
    captured once as a CUDA graph and replayed; tokens/s of the whole job."""
    import torch.nn.functional as F
    from convert_to_quant_quip_int8_b200 import ops, sharding
    from convert_to_quant_quip_int8_b200.comfy.quant_ops import QuantizedTensor
    from convert_to_quant_quip_int8_b200.stack import STACKS, LinearStack, ops_per_forward

    name = args.workload.split("_")[0]
    cfg = STACKS[name]
    rank, world, local = dist_init()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    shard = args.shard if args.shard != "auto" else "tokens"
    if world == 1:
        shard = "replica"
    st = LinearStack(name, device, rank, world, shard, chunks=args.chunks, gather=args.gather)
    warm = max(3, args.warmup)
    for _ in range(2):
        st.forward()
    torch.cuda.synchronize(device)
    ops.device_status()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        st.forward()
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize(device)
    ms, clocks = timed_region(graph.replay, args.steps, world, device)
    ops.device_status()
    ms_step = ms / args.steps
    tokens = cfg["tokens"]
    value = (world if shard == "replica" else 1) * tokens * args.steps / (ms / 1e3)
    fwd_ops = ops_per_forward(cfg["specs"]())

    # GEMM kernel time: one eager forward with CUDA events around every linear's GEMM launches
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in st.specs]
    barrier(world)
    st.forward(evs)
    torch.cuda.synchronize(device)
    gemm_ms = sum(a.elapsed_time(b) for a, b in evs)
    gemm_ms = max_over_ranks(gemm_ms, world, device)
    achieved = st.gemm_ops_local() / (gemm_ms / 1e3) / 1e12

    # e2e through the public API: host inputs -> F.linear(x, QuantizedTensor) per linear -> host output
    layout = "TensorWiseINT8Layout" if cfg["quip"] else "AxisWiseINT8Layout"
    e2e_ws = None
    if st.sharded:
        if args.gather == "peer":
            max_tn = max(s.tokens * s.n for s in st.specs)
            e2e_ws = sharding.PeerWorkspace(max_tn * 2, world, rank, device=device)
        layers = [sharding.ColumnShardedW8A8Linear.from_local(q, sc, b, world, chunks=args.chunks, peer=e2e_ws)
                  for q, sc, b in st.weights]
        apply = lambda i, x: layers[i](x)
    else:
        qts = [QuantizedTensor(q, layout, {"scale": sc if not cfg["quip"] else sc.reshape(-1, 1),
                                           "orig_dtype": torch.bfloat16}) for q, sc, _ in st.weights]
        apply = lambda i, x: F.linear(x, qts[i], st.weights[i][2])
    host_in = st.host_inputs()
    consumed = {t.src for t in st.specs if t.src != "x"}  # outputs a later linear reads
    last = st.specs[-1]
    y_host = torch.empty(last.tokens, last.n, dtype=torch.bfloat16).pin_memory()

    # host inputs in order of first use, copied on their own stream so that
    # each one overlaps the linears before it (a step's copies start after
    # the previous step's work, and a linear waits for its own input only)
    first_use = []
    for s in st.specs:
        if s.src == "x" and (s.tokens, s.k) not in first_use:
            first_use.append((s.tokens, s.k))
    copy_stream = torch.cuda.Stream(device)

    def e2e_forward():
        cur = torch.cuda.current_stream(device)
        copy_stream.wait_stream(cur)
        dev_in, ready = {}, {}
        with torch.cuda.stream(copy_stream):
            for k in first_use:
                dev_in[k] = host_in[k].to(device, non_blocking=True)
                ready[k] = torch.cuda.Event()
                ready[k].record(copy_stream)
        kept, y = {}, None
        for i, s in enumerate(st.specs):
            if s.src == "x":
                key = (s.tokens, s.k)
                if key in ready:
                    cur.wait_event(ready.pop(key))
                    dev_in[key].record_stream(cur)
                x = dev_in[key]
            else:
                x = F.gelu(kept.pop(s.src))
            y = apply(i, x)
            if s.name in consumed:
                kept[s.name] = y
        y_host.copy_(y, non_blocking=True)

    e2e_forward()
    torch.cuda.synchronize(device)
    e_steps = max(2, min(args.steps, 5))
    barrier(world)
    e2e_ms = max_over_ranks(event_time(e2e_forward, e_steps, device), world, device)
    e2e_value = (world if shard == "replica" else 1) * tokens / (e2e_ms / 1e3)
    h2d = sum(v.numel() * v.element_size() for v in host_in.values())
    ops.device_status()
    del graph
    if e2e_ws is not None:
        e2e_ws.close()
    launches = st.launches_per_forward() * args.steps
    st.close()
    if rank != 0:
        finish(world)
        return
    peak, peak_note = int8_peak()
    parallelism = {
        "columns": (f"column-sharded x{world}, output gather fused into the GEMM epilogue (peer stores over NVLink "
                    "+ peer barrier)" if args.gather == "peer" else
                    f"column-sharded x{world}, {args.chunks} token chunks, NCCL all-gather"),
        "tokens": f"token split x{world} (full weights per rank, 1/{world} of every linear's tokens, no exchange)",
        "replica": f"replicas x{world}" if world > 1 else "single GPU",
    }[shard]
    line = {
        "metric": f"{name} W8A8 linear-stack tokens/s", "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": warm, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak" if shard == "replica" else "strong", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 (fp32 epilogue, bf16 out)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations"
                + (", 1% Student-t(3) outlier channels)" if name == "t5" else ")"),
        "config": {"workload": cfg["describe"], "tokens_per_forward": tokens, "linears": len(st.specs),
                   "ops_per_forward": fwd_ops,
                   "tops": round(fwd_ops * (world if shard == "replica" else 1) / (ms_step / 1e3) / 1e12, 1),
                   "parallelism": parallelism, "graph": "one CUDA graph per forward",
                   "l2": "inputs larger than L2: every forward streams 8.6 GB (flux) / 4.6 GB (t5) of int8 weights"},
        "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(last.tokens * last.n * 2), "ms_per_step": round(e2e_ms, 3),
                "path": (f"ColumnShardedW8A8Linear ({args.gather} gather) per linear" if st.sharded
                         else f"F.linear(x, QuantizedTensor[{layout}]) per linear")
                        + ", pinned host in/out, input copies on a copy stream in order of first use"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
                     "frac": round(achieved / peak, 4), "traffic": PROFILED_TRAFFIC.get(name),
                     "traffic_basis": "ncu DRAM bytes of one single-block linear1 GEMM launch (4608 x 3072 -> 21504)"
                                      if name == "flux" else "ncu DRAM bytes of one wi GEMM launch",
                     "kernel": "gemm_pair_kernel<false,false> (per-row scales; CUDA events around every GEMM of one "
                               "eager forward" + (", incl. its peer stores)" if st.sharded and args.gather == "peer"
                                                  else ")"),
                     "algorithmic": "2 * tokens * in * out ops per linear, summed over this rank's linears",
                     "peak_note": peak_note, "gemm_ms_per_forward": round(gemm_ms, 3)},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        cv, fwd_s, threads, kind, sample = cpu_stack_baseline(name)
        line["cpu_baseline"] = cpu_baseline_field(cv, "tokens/s", threads, kind, sample, fwd_s)
    print(json.dumps(line), flush=True)
    finish(world)


def main_dit_mlp(args):
    """Config 2: the DiT MLP pair with block-128 K scales, 4096 tokens:
    K1 -> W1 block GEMM -> K1 with fused GELU -> W2 block GEMM -> bf16."""
    from convert_to_quant_quip_int8_b200 import _lib as L
    from convert_to_quant_quip_int8_b200 import ops
    from convert_to_quant_quip_int8_b200.comfy.quant_ops import QuantizedTensor
    from convert_to_quant_quip_int8_b200.workloads import DitMlpPair

    rank, world, local = dist_init()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    wl = DitMlpPair()
    su, sv = wl.w1_signs()
    q1, s1, _ = ops.quip_convert(wl.w1().to(device), su, sv, requant=L.QI8_REQ_BLOCK, want_dequant=False)
    q2, s2 = ops.requant_weight(wl.w2().to(device), L.QI8_REQ_BLOCK)
    s1, s2 = s1.reshape(q1.shape[0], -1).contiguous(), s2.reshape(q2.shape[0], -1).contiguous()
    x_cpu = wl.activations()
    T, H, F_ = wl.tokens, wl.hidden, wl.ffn
    x = x_cpu.to(device)
    stream = torch.cuda.current_stream(device)
    xq = torch.empty((T, H), dtype=torch.int8, device=device)
    xs = torch.empty((T, 1), dtype=torch.float32, device=device)
    h = torch.empty((T, F_), dtype=torch.bfloat16, device=device)
    hq = torch.empty((T, F_), dtype=torch.int8, device=device)
    hs = torch.empty((T, 1), dtype=torch.float32, device=device)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=device)
    lib = L.load()
    sp = L.stream_ptr(device)

    def k1(src, n, dst_q, dst_s, mode=L.QI8_Q_TOKEN):
        L.check(lib.qi8_quant_rows(L.ptr(src), L.QI8_BF16, T, n, n, mode, 128, L.ptr(dst_q), n, L.ptr(dst_s), sp))

    def gemm(a, a_s, b, b_s, out):
        M, K = a.shape
        N = b.shape[0]
        L.check(lib.qi8_gemm_i8(L.ptr(a), L.ptr(b), M, N, K, L.ptr(a_s), L.QI8_S_ROW, L.ptr(b_s),
                                L.QI8_S_ROW_KBLOCK, None, 0, L.ptr(out), L.QI8_BF16, N, L.QI8_ACT_NONE, sp))

    def step(ev=None):
        k1(x, H, xq, xs)
        if ev:
            ev[0].record(stream)
        gemm(xq, xs, q1, s1, h)
        if ev:
            ev[1].record(stream)
        k1(h, F_, hq, hs, L.QI8_Q_TOKEN | L.QI8_Q_GELU)  # GELU fused into the per-token quantization
        if ev:
            ev[2].record(stream)
        gemm(hq, hs, q2, s2, y)
        if ev:
            ev[3].record(stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)
    ops.device_status()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    it = iter(evs)
    ms, clocks = timed_region(lambda: step(next(it)), args.steps, world, device)
    ops.device_status()
    g1 = [e[0].elapsed_time(e[1]) for e in evs]
    g2 = [e[2].elapsed_time(e[3]) for e in evs]
    ops_step = wl.ops_per_step()
    value = world * ops_step * args.steps / (ms / 1e3) / 1e12

    w1_qt = QuantizedTensor(q1, "BlockWiseINT8Layout", {"scale": s1.reshape(F_, -1, 1), "block_size": 128,
                                                        "is_weight": True, "orig_dtype": torch.bfloat16})
    w2_qt = QuantizedTensor(q2, "BlockWiseINT8Layout", {"scale": s2.reshape(H, -1, 1), "block_size": 128,
                                                        "is_weight": True, "orig_dtype": torch.bfloat16})
    x_host = x_cpu.pin_memory()
    y_host = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        xd = x_host.to(device, non_blocking=True)
        hd = torch.nn.functional.gelu(torch.nn.functional.linear(xd, w1_qt))
        y_host.copy_(torch.nn.functional.linear(hd, w2_qt), non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier(world)
    e2e_ms = max_over_ranks(event_time(e2e_step, max(3, min(args.steps, 10)), device), world, device)
    e2e_value = world * ops_step / (e2e_ms / 1e3) / 1e12
    if rank != 0:
        finish(world)
        return
    peak, peak_note = int8_peak()
    g_avg = statistics.mean(g1 + g2)
    achieved = (2 * T * H * F_) / (g_avg / 1e3) / 1e12
    line = {
        "metric": "W8A8 QuIP linear TOPS (DiT MLP pair, block-128 K scales)", "value": round(value, 2),
        "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 (fp32 promote, bf16 out)",
        "data": "synthetic (seeded N(0,1) activations with 0.5% x30 outlier channels; N(0,0.02) weights)",
        "config": {"workload": "dit_mlp_pair_block128: x[4096,3072] bf16 -> W1[12288,3072] int8 (QuIP-rotated, "
                               "block-128 requant [12288,24,1]) + GELU -> W2[3072,12288] int8 (block-128 requant)",
                   "tokens": T, "hidden": H, "ffn": F_, "block": 128,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2: per-step footprint ~280 MB > 126 MB"},
        "e2e": {"value": round(e2e_value, 2), "unit": "TOPS", "h2d_bytes_per_step": int(T * H * 2),
                "d2h_bytes_per_step": int(T * H * 2), "ms_per_step": round(e2e_ms, 4),
                "path": "F.linear(x, QuantizedTensor W1) -> F.gelu -> F.linear(., W2), pinned host in/out"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
                     "frac": round(achieved / peak, 4), "traffic": PROFILED_TRAFFIC.get("dit_mlp"),
                     "kernel": "gemm_pair_kernel<PROMOTE,SWAP> (both GEMMs, CUDA events on the launch stream)",
                     "algorithmic": "2 * 4096 * 3072 * 12288 ops per GEMM", "peak_note": peak_note,
                     "per_gemm_ms": {"w1": round(statistics.mean(g1), 4), "w2": round(statistics.mean(g2), 4)}},
        "gpu_launches": 4 * args.steps, "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        v, unit, sec, threads, kind, sample = cpu_point("dit_mlp")
        line["cpu_baseline"] = cpu_baseline_field(v, unit, threads, kind, sample, sec)
    print(json.dumps(line), flush=True)
    finish(world)


def main_quip_linear(args):
    """Config 1: one QuIP W8A8 linear in transformed storage (tensorwise
    scale): x [512, 4096] -> K1 (signs + FWHT + per-token int8) -> K2 (int8
    GEMM, fp32 out; split over K when its tiles fill few SMs and K is long) -> K3 (FWHT +
    signs + bias -> bf16).  The step is captured once as a CUDA graph."""
    from convert_to_quant_quip_int8_b200 import _lib as L
    from convert_to_quant_quip_int8_b200 import ops
    from convert_to_quant_quip_int8_b200.comfy.quant_ops import quip_hadamard_weight
    from convert_to_quant_quip_int8_b200.workloads import SingleQuipLinear

    rank, world, local = dist_init()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    wl = SingleQuipLinear()
    su, sv = wl.signs()
    q, s, _ = ops.quip_convert(wl.weight().to(device), su, sv, store_transformed=True, want_dequant=False)
    su_d, sv_d = su.to(device), sv.to(device)
    x = wl.activations().to(device)
    bias = wl.bias().to(device)
    T, D = wl.tokens, wl.dim
    xq = torch.empty((T, D), dtype=torch.int8, device=device)
    kk = {}

    def k1():
        kk["xq"], kk["xs"] = ops.rotate_quant_rows(x, sv_d, D)

    def k2():
        kk["yh"] = ops.gemm_i8(kk["xq"], q, kk["xs"], L.QI8_S_ROW, s, L.QI8_S_ROW, None, torch.float32)

    def k3():
        kk["y"] = ops.unrotate_rows(kk["yh"], su_d, D, bias, torch.bfloat16)

    def step():
        k1(), k2(), k3()

    for _ in range(3):
        step()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    warm = max(3, args.warmup)
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize(device)
    ms, clocks = timed_region(graph.replay, args.steps, world, device)
    ops.device_status()
    # each kernel alone: a graph of it replayed 200 times between CUDA events
    # (this 12 MB working set stays in L2, as it does inside the step)
    per = {}
    for name, fn in (("k1", k1), ("k2", k2), ("k3", k3)):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        per[name] = event_time(g.replay, 200, device)
        del g
    ops_step = 2 * T * D * D
    value = world * ops_step * args.steps / (ms / 1e3) / 1e12
    split = ops._gemm_ws_bytes(T, D, D, L.QI8_S_ROW, L.QI8_S_ROW) > 0
    del graph

    # e2e: F.linear on the QuIP-Hadamard layout weight, pinned host x in, bf16 y out
    wq = quip_hadamard_weight(q, s, su_d, sv_d, D, D)
    x_host = wl.activations().pin_memory()
    y_host = torch.empty((T, D), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        y_host.copy_(torch.nn.functional.linear(x_host.to(device, non_blocking=True), wq, bias), non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier(world)
    e2e_ms = max_over_ranks(event_time(e2e_step, max(10, args.steps), device), world, device)
    if rank != 0:
        finish(world)
        return
    peak, peak_note = int8_peak()
    hbm, hbm_note = hbm_peak()
    gemm_tops = ops_step / (per["k2"] / 1e3) / 1e12
    k1_bytes = T * D * 2 + T * D + T * 4 + D * 4
    line = {
        "metric": "QuIP W8A8 rotated linear TOPS (transformed storage, tensorwise scale)",
        "value": round(value, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": warm,
        "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 (fp32 epilogue, bf16 out)",
        "data": "synthetic (seeded: W N(0,0.02), x N(0,1) with 40 outlier channels x20)",
        "config": {"workload": "quip_linear: x[512,4096] bf16, W'[4096,4096] int8 + per-row scale, signs 4096+4096",
                   "tokens": T, "dim": D, "graph": "one CUDA graph per step",
                   "l2": "inputs fit in L2 (~25 MB): L2-resident steady state"},
        "e2e": {"value": round(ops_step / (e2e_ms / 1e3) / 1e12 * world, 2), "unit": "TOPS",
                "h2d_bytes_per_step": T * D * 2, "d2h_bytes_per_step": T * D * 2, "ms_per_step": round(e2e_ms, 4),
                "path": "F.linear(x, QuantizedTensor[QuIPHadamardINT8Layout]), pinned host in/out"},
        "roofline": {"bound": "tensor", "achieved": round(gemm_tops, 1), "peak": round(peak, 1), "unit": "TOPS",
                     "frac": round(gemm_tops / peak, 4), "traffic": None,
                     "kernel": "gemm_pair_kernel (K2 alone, replayed graph)" + (" + split-K reduce" if split else ""),
                     "algorithmic": "2 * 512 * 4096 * 4096 ops", "peak_note": peak_note,
                     "whole_linear_frac": round(value / world / peak, 4),
                     "k1_rot2": {"us": round(per["k1"] * 1e3, 2), "bytes": k1_bytes,
                                 "gbs": round(k1_bytes / (per["k1"] / 1e3) / 1e9, 1),
                                 "frac_hbm": round(k1_bytes / (per["k1"] / 1e3) / 1e9 / hbm, 4),
                                 "note": "K1 = signs + FWHT + per-token int8 of x [512, 4096]; L2-resident, "
                                         "so this fraction of HBM is not an HBM measurement"},
                     "k3_us": round(per["k3"] * 1e3, 2)},
        "gpu_launches": (4 if split else 3) * args.steps, "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        v, unit, sec, threads, kind, sample = cpu_point("quip_linear", steps=3)
        line["cpu_baseline"] = cpu_baseline_field(v, unit, threads, kind, sample, sec)
    print(json.dumps(line), flush=True)
    finish(world)


def main_conversion(args):
    """Config 5: the QuIP conversion sweep (304 tensors, 12.9 B params).
    Tensors are partitioned over ranks by longest-processing-time on the
    padded size (no collective); each rank's bf16 weights are resident in
    HBM before the timed region; one step converts all of this rank's
    tensors (two-sided FWHT, rotated RTN, inverse, per-row tensorwise
    requant, then block-128 requant of the same dequantized weight)."""
    from convert_to_quant_quip_int8_b200 import _lib as L
    from convert_to_quant_quip_int8_b200 import ops, sharding
    from convert_to_quant_quip_int8_b200.workloads import conversion_sweep_tensors

    rank, world, local = dist_init()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    tensors = conversion_sweep_tensors()
    shapes = [(m, n) for _, m, n in tensors]
    mine = sharding.plan_partition(shapes, world)[rank]
    gen = torch.Generator(device=device)
    weights, signs = [], []
    for i in mine:
        m, n = shapes[i]
        gen.manual_seed(50 + i)
        weights.append((torch.randn(m, n, generator=gen, device=device) * 0.02).to(torch.bfloat16))
        mp, np_ = 1 << (m - 1).bit_length(), 1 << (n - 1).bit_length()
        gen.manual_seed(1000 + i)
        signs.append(((torch.randint(0, 2, (mp,), generator=gen, device=device) * 2 - 1).float(),
                      (torch.randint(0, 2, (np_,), generator=gen, device=device) * 2 - 1).float()))
    max_ws = max(ops.quip_workspace_bytes(*shapes[i]) for i in mine)
    ws = torch.empty(max_ws, dtype=torch.uint8, device=device)
    max_mn = max(shapes[i][0] * shapes[i][1] for i in mine)
    max_m = max(shapes[i][0] for i in mine)
    qrow = torch.empty(max_mn, dtype=torch.int8, device=device)
    qblk = torch.empty(max_mn, dtype=torch.int8, device=device)
    srow = torch.empty(max_m, dtype=torch.float32, device=device)
    sblk = torch.empty(max_mn // 128, dtype=torch.float32, device=device)
    lib = L.load()

    def convert_one(w, su, sv, sp):
        M, N = w.shape
        L.check(lib.qi8_quip_convert(L.ptr(w), L.QI8_BF16, M, N, L.ptr(su), L.ptr(sv), 0, L.QI8_REQ_ROW, 128,
                                     L.ptr(qrow), L.ptr(srow), None, L.ptr(ws), ws.numel(), sp), "qi8_quip_convert")
        # the dequantized weight is left in the workspace plane (fp32, row stride N_pad)
        L.check(lib.qi8_requant_weight(L.ptr(ws), L.QI8_F32, M, N, 1 << (N - 1).bit_length(), L.QI8_REQ_BLOCK,
                                       128, L.ptr(qblk), L.ptr(sblk), None, 0, sp), "qi8_requant_weight")

    def step():
        sp = L.stream_ptr(device)
        for w, (su, sv) in zip(weights, signs):
            convert_one(w, su, sv, sp)

    step()
    torch.cuda.synchronize(device)
    steps = max(1, min(args.steps, 5))
    ms, clocks = timed_region(step, steps, world, device)
    ops.device_status()
    params = sum(m * n for m, n in shapes)
    value = len(shapes) * steps / (ms / 1e3)
    my_params = sum(shapes[i][0] * shapes[i][1] for i in mine)

    # e2e: pinned host bf16 weights -> device -> conversion -> pinned host int8 (both requants) + scales;
    # one pinned host tensor per distinct shape stands in for every tensor of that shape
    host_w, host_q = {}, {}
    for i in mine:
        shp = shapes[i]
        if shp not in host_w:
            host_w[shp] = (torch.randn(*shp, generator=_gen(60 + len(host_w))) * 0.02).to(torch.bfloat16).pin_memory()
            host_q[shp] = (torch.empty(shp[0] * shp[1] * 2, dtype=torch.int8).pin_memory(),
                           torch.empty(shp[0] * (1 + shp[1] // 128), dtype=torch.float32).pin_memory())
    wdev = torch.empty(max_mn, dtype=torch.bfloat16, device=device)
    h2d = d2h = 0

    def e2e_step():
        nonlocal h2d, d2h
        h2d = d2h = 0
        sp = L.stream_ptr(device)
        for k, i in enumerate(mine):
            M, N = shapes[i]
            w = wdev[: M * N].view(M, N)
            w.copy_(host_w[(M, N)], non_blocking=True)
            convert_one(w, signs[k][0], signs[k][1], sp)
            hq, hs = host_q[(M, N)]
            hq[: M * N].copy_(qrow[: M * N], non_blocking=True)
            hq[M * N:].copy_(qblk[: M * N], non_blocking=True)
            hs[:M].copy_(srow[:M], non_blocking=True)
            hs[M:].copy_(sblk[: M * N // 128], non_blocking=True)
            h2d += M * N * 2
            d2h += 2 * M * N + 4 * (M + M * N // 128)

    e2e_step()
    barrier(world)
    e2e_ms = max_over_ranks(event_time(e2e_step, 1, device), world, device)
    del ws
    if rank != 0:
        finish(world)
        return
    hbm, hbm_note = hbm_peak()
    min_bytes = 4 * my_params  # bf16 read + int8 per-row + int8 block writes

    def launches(m):  # column passes (one up to 2^9 rows, else two) forward and inverse, row pass, two requants
        col = 1 if (1 << (m - 1).bit_length()) <= 512 else 2
        return 2 * col + 3
    achieved = min_bytes / (ms / steps / 1e3) / 1e9
    line = {
        "metric": "QuIP conversion sweep tensors/s (304 tensors, 12.9 B params)", "value": round(value, 2),
        "unit": "tensors/s", "n_gpus": world, "steps": steps, "warmup": 1, "ms_per_step": round(ms / steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32 transform, int8 out",
        "weight_gb_per_s": round(params * 2 * steps / (ms / 1e3) / 1e9, 1),
        "data": "synthetic (seeded N(0,0.02) bf16 weights resident in HBM)",
        "config": {"workload": "conversion_sweep: 304 tensors, two-sided FWHT + rotated RTN + inverse + per-row "
                               "and block-128 requant, LPT partition by padded size",
                   "params": params, "parallelism": f"tensor-partitioned x{world}" if world > 1 else "single GPU"},
        "e2e": {"value": round(len(shapes) / (e2e_ms / 1e3), 2), "unit": "tensors/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 2),
                "path": "pinned host bf16 -> device -> qi8_quip_convert + qi8_requant_weight -> pinned host int8"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(hbm, 1), "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None,
                     "algorithmic": "4 B per parameter (bf16 read, int8 per-row and int8 block writes)",
                     "kernel": "whole conversion step (column/row FWHT passes, RTN, inverse, requants)",
                     "peak_note": hbm_note},
        "gpu_launches": steps * sum(launches(shapes[i][0]) for i in mine), "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        v, unit, sec, threads, kind, sample = cpu_point("conversion")
        line["cpu_baseline"] = cpu_baseline_field(v, unit, threads, kind, sample, sec)
    print(json.dumps(line), flush=True)
    finish(world)


LDLQ_METRIC = "QuIP default-converter tensors/s (one Flux double + single block, 10 tensors, 0.34 B params)"
FP64_TFLOPS = 37.2  # fp64 tensor-core (mma.sync f64) rate of a register-only loop on this pool's B200


def ldlq_launches(m: int, n: int) -> int:
    """libqi8 kernel launches of one default conversion (diagonal rescaling,
    per-row requant) of an [m, n] weight."""
    mp, np_ = 1 << (m - 1).bit_length(), 1 << (n - 1).bit_length()
    colp = lambda rows: 1 if rows <= 512 else 2  # column FWHT passes
    leaves = max(1, np_ // 64)  # recursive Cholesky-inverse: 64-wide leaves, 4 GEMMs per inner node
    hinv = leaves + 4 * (leaves - 1) + 1
    nbk = (np_ + 127) // 128
    return (1 + 2 + (colp(mp) + 1) + (colp(np_) + 1) + 2 + hinv + (2 * nbk - 1) + 1 + (1 + colp(mp)) + 1 + 1)


def main_conversion_ldlq(args):
    """The converter with the reference's defaults (QuIPInt8Converter(seed),
    converters/quip_int8.py:1031-1669) on the 10 weights of one Flux double
    and one single block, bf16 resident in HBM; one step converts all ten
    (per-row tensorwise requant).  Tensors are partitioned over ranks like
    the conversion sweep (no collective)."""
    from convert_to_quant_quip_int8_b200 import ops, sharding
    from convert_to_quant_quip_int8_b200.converters.quip_int8 import QuIPInt8Converter
    from convert_to_quant_quip_int8_b200.workloads import ldlq_block_tensors

    rank, world, local = dist_init()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    shapes = [(m, n) for _, m, n in ldlq_block_tensors()]
    mine = sharding.plan_partition(shapes, world)[rank]
    gen = torch.Generator(device=device)
    weights = []
    for i in mine:
        gen.manual_seed(70 + i)
        weights.append((torch.randn(*shapes[i], generator=gen, device=device) * 0.02).to(torch.bfloat16))
    conv = QuIPInt8Converter(seed=1000, device=str(device))

    def step():
        for w in weights:
            conv.convert(w)

    step()
    torch.cuda.synchronize(device)
    steps = max(1, min(args.steps, 3))
    ms, clocks = timed_region(step, steps, world, device)
    ops.device_status()
    value = len(shapes) * steps / (ms / 1e3)
    params = sum(m * n for m, n in shapes)

    # the dominant kernels (the fp64 factorization) timed live with CUDA events on one more step
    hinv_times = {}
    orig = ops.hinv_upper

    def timed_hinv(h_rev):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        out = orig(h_rev)
        b.record()
        hinv_times.setdefault(h_rev.shape[0], []).append((a, b))
        return out

    ops.hinv_upper = timed_hinv
    try:
        step()
    finally:
        ops.hinv_upper = orig
    torch.cuda.synchronize(device)
    step_ms = ms / steps
    fact_ms = sum(a.elapsed_time(b) for v in hinv_times.values() for a, b in v)
    nbig = max(hinv_times) if hinv_times else 0
    big = [a.elapsed_time(b) for a, b in hinv_times.get(nbig, [])]

    # e2e: pinned host bf16 -> device -> converter -> pinned host int8 + scales
    host_w = [w.cpu().pin_memory() for w in weights]
    host_q = [(torch.empty(w.shape, dtype=torch.int8).pin_memory(),
               torch.empty((w.shape[0], 1), dtype=torch.float32).pin_memory()) for w in weights]
    h2d = d2h = 0

    def e2e_step():
        nonlocal h2d, d2h
        h2d = d2h = 0
        for hw, (hq, hs) in zip(host_w, host_q):
            w = hw.to(device, non_blocking=True)
            q, s = conv.convert(w)[:2]
            hq.copy_(q, non_blocking=True)
            hs.copy_(s.reshape(hs.shape), non_blocking=True)
            h2d += hw.numel() * 2
            d2h += hq.numel() + hs.numel() * 4

    e2e_step()
    barrier(world)
    e2e_ms = max_over_ranks(event_time(e2e_step, 1, device), world, device)
    if rank != 0:
        finish(world)
        return
    achieved = (2.0 / 3.0) * nbig ** 3 / (statistics.mean(big) / 1e3) / 1e12 if big else None
    line = {
        "metric": LDLQ_METRIC, "value": round(value, 3), "unit": "tensors/s", "n_gpus": world, "steps": steps,
        "warmup": 1, "ms_per_step": round(step_ms, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp64 factorization, fp32 LDLQ, int8 out",
        "weight_gb_per_s": round(params * 2 / (step_ms / 1e3) / 1e9, 2),
        "data": "synthetic (seeded N(0,0.02) bf16 weights resident in HBM)",
        "config": {"workload": "QuIPInt8Converter defaults (diagonal rescaling, random permutation, act-order, "
                               "damping, fp64 Hessian factorization, blocked LDLQ, per-row requant), H = identity, "
                               "Flux double block (img + txt: qkv, proj, mlp0, mlp2) + single block "
                               "(linear1, linear2)", "params": params,
                   "parallelism": f"tensor-partitioned x{world}" if world > 1 else "single GPU"},
        "e2e": {"value": round(len(shapes) / (e2e_ms / 1e3), 3), "unit": "tensors/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 2),
                "path": "pinned host bf16 -> device -> QuIPInt8Converter.convert -> pinned host int8 + scales"},
        "roofline": {"bound": "fp64", "achieved": round(achieved, 2) if achieved else None,
                     "peak": FP64_TFLOPS, "unit": "TFLOP/s",
                     "frac": round(achieved / FP64_TFLOPS, 4) if achieved else None, "traffic": None,
                     "algorithmic": f"2/3 N^3 fp64 flops per factorization (Cholesky N^3/3 + triangular inverse "
                                    f"N^3/3), N = {nbig}",
                     "kernel": "qi8_hinv_upper (potf2_inv_kernel + dgemm_mma_kernel launches)",
                     "share_of_step": round(fact_ms / step_ms, 3),
                     "peak_note": "fp64 tensor-core ceiling measured by a register-only mma.sync f64 loop "
                                  "(37.2 TF/s; SIMT DFMA 33.9); no fp64 figure in MEASURED_PEAKS.json"},
        "gpu_launches": steps * sum(ldlq_launches(*shapes[i]) for i in mine), "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        v, unit, sec, threads, kind, sample = cpu_point("conversion_ldlq")
        line["cpu_baseline"] = cpu_baseline_field(v, unit, threads, kind, sample, sec)
    print(json.dumps(line), flush=True)
    finish(world)


# ======================================================= reference arm
def main_reference(args):
    """The reference's CPU path on this box's host cores (rank 0 only), on
    this framework's metric, unit and config."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    wl = args.workload
    if wl in ("flux_stack", "t5_stack"):
        from convert_to_quant_quip_int8_b200.stack import STACKS
        name = wl.split("_")[0]
        threads = cpu_threads()
        st = StackCPU(name)
        keys = list(st.counts)
        first = keys[0]
        st.run(first)
        st.times[first].clear()
        # warm-up and timed steps each run one distinct linear shape, round robin;
        # every shape is timed at least once
        for i in range(max(0, args.warmup)):
            st.run(keys[i % len(keys)])
        for k in keys:
            st.times[k].clear()
        for i in range(max(len(keys), args.steps)):
            st.run(keys[i % len(keys)])
        fwd = st.forward_seconds()
        value, unit, metric = st.cfg["tokens"] / fwd, "tokens/s", f"{name} W8A8 linear-stack tokens/s"
        config = {"workload": STACKS[name]["describe"], "parallelism": "cpu"}
        scaling = "weak" if args.shard == "replica" else "strong"
        kind, sample, ms_step = st.kind, st.sample(), fwd * 1e3
    else:
        steps = max(1, min(args.steps, 5))
        value, unit, sec, threads, kind, sample = cpu_point(wl, steps=steps, warmup=min(args.warmup, 1))
        metric = {"dit_mlp": "W8A8 QuIP linear TOPS (DiT MLP pair, block-128 K scales)",
                  "quip_linear": "QuIP W8A8 rotated linear TOPS (transformed storage, tensorwise scale)",
                  "conversion": "QuIP conversion sweep tensors/s (304 tensors, 12.9 B params)",
                  "conversion_ldlq": LDLQ_METRIC}[wl]
        config = {"workload": wl, "parallelism": "cpu"}
        scaling = "strong" if wl.startswith("conversion") else "weak"
        ms_step = sec * 1e3
    line = {"impl": "reference", "metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 2),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "int8 x int8 -> int32 (fp32 epilogue)", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return main_reference(args)
    if args.workload in ("flux_stack", "t5_stack"):
        return main_stack(args)
    if args.workload == "dit_mlp":
        return main_dit_mlp(args)
    if args.workload == "quip_linear":
        return main_quip_linear(args)
    if args.workload == "conversion_ldlq":
        return main_conversion_ldlq(args)
    return main_conversion(args)


if __name__ == "__main__":
    main()
