"""Benchmark of the QuIP W8A8 quantized-linear path on B200.

Workload (one step): the DiT MLP pair with block-128 K scales --
x [4096, 3072] bf16 -> per-token int8 (K1) -> W1 [12288, 3072] int8 GEMM with
per-128-K-block promotion (K2) -> GELU + per-token int8 (K1) ->
W2 [3072, 12288] int8 GEMM (K2) -> bf16 [4096, 3072].
Metric: W8A8 linear TOPS (2 * M * N * K per GEMM, both GEMMs), whole job.

    python bench.py [--gpus N --steps K --warmup W]          # this framework
    python bench.py --impl reference [...]                     # CPU reference arm

Multi-GPU (torchrun, one rank per GPU): every rank runs its own replica of
the workload (weak scaling, no collective on the data path); the time is
the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = ("dit_mlp_pair_block128: x[4096,3072] bf16 -> W1[12288,3072] int8 (QuIP-rotated, block-128 requant "
            "[12288,24,1]) + GELU -> W2[3072,12288] int8 (block-128 requant) -> bf16")
METRIC = "W8A8 QuIP linear TOPS (DiT MLP pair, block-128 K scales)"
UNIT = "TOPS"
L2_NOTE = "inputs larger than L2: per-step footprint ~280 MB (x 25 MB, W1+W2 75 MB, h 100 MB + 50 MB, y 25 MB) > 126 MB"


PROFILE_GEMM = os.path.join(ROOT, "profiles", "gemm_pair_kernel_block_dit_mlp.md")


def profiled_traffic():
    """DRAM bytes per GEMM launch (dram__bytes_read.sum + dram__bytes_write.sum,
    averaged over the W1 and W2 launches) from the committed ncu summary of
    this workload, or None when the summary is absent."""
    try:
        with open(PROFILE_GEMM) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="qi8", choices=["qi8", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=512, help="token sample of the CPU baseline step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="dit_mlp",
                    choices=["dit_mlp", "quip_linear", "conversion", "flux_stack", "t5_stack"],
                    help="dit_mlp: the headline DiT MLP pair; quip_linear: one rotated W8A8 linear "
                         "(K1 rotate -> K2 -> K3); conversion: the 304-tensor QuIP conversion sweep; "
                         "flux_stack / t5_stack: the 228-linear Flux-shaped / 168-linear T5-XXL stacks")
    ap.add_argument("--shard", default="replica", choices=["replica", "columns", "tokens"],
                    help="stacks on N>1 GPUs: replica = one batch per rank (weak scaling); columns = every "
                         "linear column-sharded with its output gathered on every rank; tokens = full weights, "
                         "each rank 1/N of the tokens (both strong scaling)")
    ap.add_argument("--chunks", type=int, default=4, help="token chunks per column-sharded linear (nccl gather)")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="column-sharded output gather: peer = fused into the GEMM epilogue (stores into every "
                         "rank's IPC-mapped buffer + peer barrier); nccl = chunked NCCL all-gather + re-layout")
    return ap.parse_args()


# ----------------------------------------------------------------- peaks
def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


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
def dist_init(n_gpus: int):
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


# ------------------------------------------------------------ CPU arm
def cpu_reference_step_fn(tokens: int):
    """One step of the CPU oracle port (numpy) on a `tokens`-row sample of the
    workload; returns (callable, ops per call, description)."""
    import oracle as O
    from convert_to_quant_quip_int8_b200.workloads import DitMlpPair

    wl = DitMlpPair()
    x = wl.activations()[:tokens].float().numpy()
    # weights: block-128 requant of the same seeded tensors (the offline
    # rotation of W1 is conversion-time work and does not change the timed step)
    q1, s1 = O.quip_requant(wl.w1().float().numpy(), "block", True)
    q2, s2 = O.quip_requant(wl.w2().float().numpy(), "block", True)
    s1 = s1.reshape(q1.shape[0], -1)
    s2 = s2.reshape(q2.shape[0], -1)

    def step():
        xq, xs = O.quantize_int8_axiswise(x)
        h = O.int8_gemm_block(xq, np.ones((tokens, 1), np.float32), q1, s1, None, b_layout="row") * xs
        h = O.round_bf16(O.gelu_f32(O.round_bf16(h)))
        hq, hs = O.quantize_int8_axiswise(h)
        y = O.int8_gemm_block(hq, np.ones((tokens, 1), np.float32), q2, s2, None, b_layout="row") * hs
        return O.f32_to_bf16(y)

    return step, wl.ops_per_step(tokens), f"{tokens} of 4096 tokens through both linears (numpy oracle port)"


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_cpu(tokens: int, steps: int, warmup: int):
    step, ops, sample = cpu_reference_step_fn(tokens)
    for _ in range(max(0, warmup)):
        step()
    times = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return ops / med / 1e12, med, sample


# ------------------------------------------------------------- GPU arm
def build_model(device):
    from convert_to_quant_quip_int8_b200 import _lib as L
    from convert_to_quant_quip_int8_b200 import ops
    from convert_to_quant_quip_int8_b200.workloads import DitMlpPair

    wl = DitMlpPair()
    x = wl.activations()
    su, sv = wl.w1_signs()
    w1 = wl.w1().to(device)
    q1, s1, _ = ops.quip_convert(w1, su, sv, requant=L.QI8_REQ_BLOCK, want_dequant=False)
    del w1
    w2 = wl.w2().to(device)
    q2, s2 = ops.requant_weight(w2, L.QI8_REQ_BLOCK)
    del w2
    torch.cuda.synchronize(device)
    return wl, x, (q1, s1.reshape(q1.shape[0], -1).contiguous()), (q2, s2.reshape(q2.shape[0], -1).contiguous())


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


def main_quip_linear(args):
    """Config 1: one QuIP W8A8 linear in transformed storage (tensorwise
    scale): x [512, 4096] -> K1 (signs + FWHT + per-token int8) -> K2 (int8
    GEMM, fp32 out; split over K when its tiles fill few SMs) -> K3 (FWHT +
    signs + bias -> bf16).  The step is captured once as a CUDA graph."""
    from convert_to_quant_quip_int8_b200 import _lib as L
    from convert_to_quant_quip_int8_b200 import ops
    from convert_to_quant_quip_int8_b200.workloads import SingleQuipLinear

    rank, world, local = dist_init(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    wl = SingleQuipLinear()
    su, sv = wl.signs()
    q, s, _ = ops.quip_convert(wl.weight().to(device), su, sv, store_transformed=True, want_dequant=False)
    su_d, sv_d = su.to(device), sv.to(device)
    x = wl.activations().to(device)
    bias = wl.bias().to(device)
    T, D = wl.tokens, wl.dim

    def step():
        xq, xs = ops.rotate_quant_rows(x, sv_d, D)
        y_had = ops.gemm_i8(xq, q, xs, L.QI8_S_ROW, s, L.QI8_S_ROW, None, torch.float32)
        return ops.unrotate_rows(y_had, su_d, D, bias, torch.bfloat16)

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
    # GEMM alone: a graph holding only K2 (and its split-K reduce), replayed
    # back to back between two CUDA events (L2 holds this small case)
    xq0, xs0 = ops.rotate_quant_rows(x, sv_d, D)
    ggraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ggraph):
        ops.gemm_i8(xq0, q, xs0, L.QI8_S_ROW, s, L.QI8_S_ROW, None, torch.float32)
    for _ in range(3):
        ggraph.replay()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    g0.record()
    for _ in range(200):
        ggraph.replay()
    g1.record()
    torch.cuda.synchronize(device)
    gemm_ms = g0.elapsed_time(g1) / 200
    del ggraph
    ops_step = 2 * T * D * D
    value = world * ops_step * args.steps / (ms / 1e3) / 1e12
    split = ops._gemm_ws_bytes(T, D, D, L.QI8_S_ROW, L.QI8_S_ROW) > 0
    del graph
    if rank == 0:
        peaks, peak_kind = measured_peaks()
        int8_peak = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
        gemm_tops = ops_step / (gemm_ms / 1e3) / 1e12
        print(json.dumps({
            "metric": "QuIP W8A8 rotated linear TOPS (transformed storage, tensorwise scale)",
            "value": round(value, 2), "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> int32 (fp32 epilogue, bf16 out)",
            "data": "synthetic (seeded: W N(0,0.02), x N(0,1) with 40 outlier channels x20)",
            "config": {"workload": "quip_linear: x[512,4096] bf16, W'[4096,4096] int8 + scalar scale, signs 4096+4096",
                       "tokens": T, "dim": D, "graph": "one CUDA graph per step",
                       "l2": "inputs fit in L2 (~25 MB): L2-resident steady state"},
            "roofline": {"bound": "tensor", "achieved": round(gemm_tops, 1), "peak": round(int8_peak, 1),
                         "unit": "TOPS", "frac": round(gemm_tops / int8_peak, 4), "traffic": None,
                         "kernel": "gemm_pair_kernel (K2 alone: a graph of it replayed 200 times between CUDA events)"
                                   + (" + split-K reduce" if split else ""),
                         "whole_linear_frac": round(value / world / int8_peak, 4),
                         "peak_note": f"dense int8 = 2 x {peak_kind} cuBLAS bf16 burst"},
            "gpu_launches": (4 if split else 3) * args.steps, "clocks": clocks}), flush=True)
    _finish(world)


def main_conversion(args):
    """Config 5: the QuIP conversion sweep (304 tensors, 12.9 B params).
    Tensors are partitioned over ranks by longest-processing-time on the
    padded size (no collective); each rank's bf16 weights are resident in
    HBM before the timed region; one step converts all of this rank's
    tensors (two-sided FWHT, rotated RTN, inverse, block-128 requant)."""
    from convert_to_quant_quip_int8_b200 import _lib as L
    from convert_to_quant_quip_int8_b200 import ops, sharding
    from convert_to_quant_quip_int8_b200.workloads import conversion_sweep_tensors

    rank, world, local = dist_init(args.gpus)
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
    qbuf = torch.empty(max_mn, dtype=torch.int8, device=device)

    def step():
        for w, (su, sv) in zip(weights, signs):
            ops.quip_convert(w, su, sv, requant=L.QI8_REQ_BLOCK, want_dequant=False, workspace=ws)
        return qbuf

    step()
    torch.cuda.synchronize(device)
    steps = max(1, args.steps)
    ms, clocks = timed_region(step, steps, world, device)
    ops.device_status()
    params = sum(shapes[i][0] * shapes[i][1] for i in range(len(shapes)))
    value = len(shapes) * steps / (ms / 1e3)  # tensors/s of the whole job
    if rank == 0:
        print(json.dumps({
            "metric": "QuIP conversion sweep tensors/s (304 tensors, 12.9 B params)",
            "value": round(value, 2), "unit": "tensors/s", "n_gpus": world, "steps": steps, "warmup": 1,
            "ms_per_step": round(ms / steps, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32 transform, int8 out",
            "weight_gb_per_s": round(params * 2 * steps / (ms / 1e3) / 1e9, 1),
            "data": "synthetic (seeded N(0,0.02) bf16 weights resident in HBM)",
            "config": {"workload": "conversion_sweep: 304 tensors, LPT partition by padded size, block-128 requant",
                       "params": params, "parallelism": f"tensor-partitioned x{world}"},
            "clocks": clocks}), flush=True)
    _finish(world)


def cpu_stack_step_fn(name: str, tokens: int = 256):
    """CPU oracle port of one linear of every distinct shape of a stack on a
    ``tokens``-row sample; returns (callable, ops per call, description)."""
    import oracle as O
    from convert_to_quant_quip_int8_b200.stack import STACKS

    cfg = STACKS[name]
    shapes = sorted({(s.k, s.n, s.gelu) for s in cfg["specs"]()})
    rng = np.random.default_rng(0)
    cases = []
    for k, n, gelu in shapes:
        x = O.round_bf16(rng.standard_normal((tokens, k)).astype(np.float32))
        wq, ws = O.quantize_int8_axiswise(O.round_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32)))
        b = O.round_bf16((rng.standard_normal(n) * 0.01).astype(np.float32)) if cfg["bias"] else None
        cases.append((x, wq, ws.reshape(-1), b, gelu))

    def step():
        for x, wq, ws, b, gelu in cases:
            xin = O.round_bf16(O.gelu_f32(x)) if gelu else x
            O.f32_to_bf16(O.linear_w8a8(xin, wq, ws, b)[3])

    ops = sum(2 * tokens * k * n for k, n, _ in shapes)
    return step, ops, (f"one linear of each of the {len(shapes)} distinct shapes at {tokens} tokens "
                       f"(numpy oracle port), scaled to the stack's ops per forward")


def run_cpu_stack(name: str, steps: int, warmup: int):
    """CPU tokens/s of the stack, extrapolated from the timed sample by ops."""
    from convert_to_quant_quip_int8_b200.stack import STACKS, ops_per_forward

    step, ops, sample = cpu_stack_step_fn(name)
    for _ in range(max(0, warmup)):
        step()
    times = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    cfg = STACKS[name]
    fwd_s = ops_per_forward(cfg["specs"]()) / (ops / med)
    return cfg["tokens"] / fwd_s, med, sample


def main_stack(args):
    """Configs 3 and 4: a whole linear stack per step (K1 + K2 per linear),
    captured once as a CUDA graph and replayed; tokens/s of the whole job."""
    import torch.nn.functional as F
    from convert_to_quant_quip_int8_b200 import _lib as L
    from convert_to_quant_quip_int8_b200 import ops, sharding
    from convert_to_quant_quip_int8_b200.comfy.quant_ops import QuantizedTensor
    from convert_to_quant_quip_int8_b200.stack import STACKS, LinearStack, ops_per_forward

    name = args.workload.split("_")[0]
    cfg = STACKS[name]
    rank, world, local = dist_init(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    shard = args.shard if world > 1 else "replica"
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
    fwd_ops = ops_per_forward(st.specs) * (world if shard == "tokens" else 1)

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
    if shard == "columns":
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
    last = st.specs[-1]
    y_host = torch.empty(last.tokens, last.n, dtype=torch.bfloat16).pin_memory()

    def e2e_forward():
        dev_in = {k: v.to(device, non_blocking=True) for k, v in host_in.items()}
        kept, y = {}, None
        for i, s in enumerate(st.specs):
            x = dev_in[(s.tokens, s.k)] if s.src == "x" else F.gelu(kept.pop(s.src))
            y = apply(i, x)
            if any(t.src == s.name for t in st.specs):
                kept[s.name] = y
        y_host.copy_(y, non_blocking=True)

    e2e_forward()
    torch.cuda.synchronize(device)
    e_steps = max(2, min(args.steps, 5))
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        e2e_forward()
    e1.record()
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, device) / e_steps
    e2e_value = (world if shard == "replica" else 1) * tokens / (e2e_ms / 1e3)
    h2d = sum(v.numel() * v.element_size() for v in host_in.values())
    ops.device_status()
    del graph
    if e2e_ws is not None:
        e2e_ws.close()
    st.close()
    if rank != 0:
        _finish(world)
        return
    peaks, peak_kind = measured_peaks()
    int8_peak = 2.0 * float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1400.0)))
    line = {
        "metric": f"{name} W8A8 linear-stack tokens/s", "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": warm, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak" if shard == "replica" else "strong", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 (fp32 epilogue, bf16 out)",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations"
                + (", 1% Student-t(3) outlier channels)" if name == "t5" else ")"),
        "config": {"workload": cfg["describe"], "tokens_per_forward": tokens, "linears": len(st.specs),
                   "ops_per_forward": fwd_ops, "tops": round(fwd_ops * (world if shard == "replica" else 1)
                                                             / (ms_step / 1e3) / 1e12, 1),
                   "parallelism": ((f"column-sharded x{world}, output gather fused into the GEMM epilogue "
                                    "(peer stores over NVLink + peer barrier)" if args.gather == "peer" else
                                    f"column-sharded x{world}, {args.chunks} token chunks, NCCL all-gather")
                                   if shard == "columns" else
                                   (f"token split x{world} (full weights per rank, no exchange)" if shard == "tokens"
                                    else (f"replicas x{world}" if world > 1 else "single"))),
                   "graph": "one CUDA graph per forward",
                   "l2": "inputs larger than L2: every forward streams 8.6 GB (flux) / 4.6 GB (t5) of int8 weights"},
        "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(last.tokens * last.n * 2), "ms_per_step": round(e2e_ms, 3),
                "path": (f"ColumnShardedW8A8Linear ({args.gather} gather) per linear" if shard == "columns"
                         else f"F.linear(x, QuantizedTensor[{layout}]) per linear") + ", pinned host in/out"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1), "unit": "TOPS",
                     "frac": round(achieved / int8_peak, 4), "traffic": None,
                     "kernel": "gemm_pair_kernel<false,false> (per-row scales; CUDA events around every GEMM "
                               "of one eager forward" + (", incl. its peer stores)" if shard == "columns" and
                                                         args.gather == "peer" else ")"),
                     "peak_note": f"dense int8 = 2 x {peak_kind} cuBLAS bf16 sustained "
                                  f"({peaks.get('bf16_tflops_sustained')} TF/s)",
                     "gemm_ms_per_forward": round(gemm_ms, 3)},
        "gpu_launches": st.launches_per_forward() * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        torch.set_num_threads(cpu_cores())
        cv, cmed, sample = run_cpu_stack(name, 2, 1)
        line["cpu_baseline"] = {"value": round(cv, 3), "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
                                "sample": sample, "s_per_sample": round(cmed, 3)}
    print(json.dumps(line), flush=True)
    _finish(world)


def main():
    args = parse()
    if args.impl == "reference":
        return main_reference(args)
    if args.workload == "quip_linear":
        return main_quip_linear(args)
    if args.workload == "conversion":
        return main_conversion(args)
    if args.workload in ("flux_stack", "t5_stack"):
        return main_stack(args)
    from convert_to_quant_quip_int8_b200 import _lib as L
    from convert_to_quant_quip_int8_b200 import ops
    from convert_to_quant_quip_int8_b200.comfy.quant_ops import QuantizedTensor

    rank, world, local = dist_init(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    wl, x_cpu, (q1, s1), (q2, s2) = build_model(device)
    T, H, F_ = wl.tokens, wl.hidden, wl.ffn
    x = x_cpu.to(device)
    stream = torch.cuda.current_stream(device)

    # preallocated activations
    xq = torch.empty((T, H), dtype=torch.int8, device=device)
    h = torch.empty((T, F_), dtype=torch.bfloat16, device=device)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=device)
    lib = L.load()
    sp = L.stream_ptr(device)

    def k1(src, n, dst_q, dst_s, mode=L.QI8_Q_TOKEN):
        L.check(lib.qi8_quant_rows(L.ptr(src), L.QI8_BF16, T, n, n, mode, 128, L.ptr(dst_q), n,
                                   L.ptr(dst_s), sp))

    xs = torch.empty((T, 1), dtype=torch.float32, device=device)
    hq = torch.empty((T, F_), dtype=torch.int8, device=device)
    hs = torch.empty((T, 1), dtype=torch.float32, device=device)

    def gemm(a, a_s, b, b_s, out, act):
        M, K = a.shape
        N = b.shape[0]
        L.check(lib.qi8_gemm_i8(L.ptr(a), L.ptr(b), M, N, K, L.ptr(a_s), L.QI8_S_ROW, L.ptr(b_s),
                                L.QI8_S_ROW_KBLOCK, None, 0, L.ptr(out), L.QI8_BF16, N, act, sp))

    def step(ev=None):
        k1(x, H, xq, xs)
        if ev:
            ev[0].record(stream)
        gemm(xq, xs, q1, s1, h, L.QI8_ACT_NONE)
        if ev:
            ev[1].record(stream)
        k1(h, F_, hq, hs, L.QI8_Q_TOKEN | L.QI8_Q_GELU)  # GELU fused into the per-token quantization
        if ev:
            ev[2].record(stream)
        gemm(hq, hs, q2, s2, y, L.QI8_ACT_NONE)
        if ev:
            ev[3].record(stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)
    ops.device_status()

    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches_per_step = 4
    # per-step events around the two GEMMs, all on the launching stream
    gemm_ms = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    with ClockProbe(device.index if device.index is not None else 0) as probe:
        barrier(world)
        torch.cuda.synchronize(device)
        t_start.record(stream)
        for i in range(args.steps):
            step(gemm_ms[i])
        t_end.record(stream)
        torch.cuda.synchronize(device)
        barrier(world)
    ops.device_status()
    elapsed_ms = t_start.elapsed_time(t_end)
    elapsed_ms = max_over_ranks(elapsed_ms, world, device)
    g1 = [e[0].elapsed_time(e[1]) for e in gemm_ms]
    g2 = [e[2].elapsed_time(e[3]) for e in gemm_ms]
    ops_step = wl.ops_per_step()
    value = world * ops_step * args.steps / (elapsed_ms / 1e3) / 1e12
    ms_per_step = elapsed_ms / args.steps

    # ---- e2e through the public API: host pinned x -> F.linear -> GELU -> F.linear -> host
    w1_qt = QuantizedTensor(q1, "BlockWiseINT8Layout", {"scale": s1.reshape(F_, -1, 1), "block_size": 128,
                                                        "is_weight": True, "orig_dtype": torch.bfloat16})
    w2_qt = QuantizedTensor(q2, "BlockWiseINT8Layout", {"scale": s2.reshape(H, -1, 1), "block_size": 128,
                                                        "is_weight": True, "orig_dtype": torch.bfloat16})
    x_host = x_cpu.pin_memory()
    y_host = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        xd = x_host.to(device, non_blocking=True)
        hd = torch.nn.functional.gelu(torch.nn.functional.linear(xd, w1_qt))
        yd = torch.nn.functional.linear(hd, w2_qt)
        y_host.copy_(yd, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(device)
    e_steps = max(3, min(args.steps, 10))
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, device) / e_steps
    e2e_value = world * ops_step / (e2e_ms / 1e3) / 1e12
    # parity spot check of the timed path against the public-API path
    ref_y = y.float()
    rel = float((y_host.to(device).float() - ref_y).norm() / ref_y.norm().clamp_min(1e-30))

    if rank != 0:
        _finish(world)
        return

    peaks, peak_kind = measured_peaks()
    int8_peak = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    gemm_ops = 2 * T * H * F_
    g_avg_ms = statistics.mean(g1 + g2)
    achieved = gemm_ops / (g_avg_ms / 1e3) / 1e12
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> int32 (fp32 promote, bf16 out)",
        "data": "synthetic (seeded N(0,1) activations with 0.5% x30 outlier channels; N(0,0.02) weights)",
        "config": {"workload": WORKLOAD, "tokens": T, "hidden": H, "ffn": F_, "block": 128,
                   "parallelism": f"replicas x{world}" if world > 1 else "single", "l2": L2_NOTE},
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": int(T * H * 2),
                "d2h_bytes_per_step": int(T * H * 2), "ms_per_step": round(e2e_ms, 4),
                "path": "F.linear(x, QuantizedTensor W1) -> F.gelu -> F.linear(., W2), pinned host in/out",
                "rel_err_vs_device_path": rel},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak, 1),
                     "unit": "TOPS", "frac": round(achieved / int8_peak, 4), "traffic": profiled_traffic(),
                     "traffic_note": "DRAM bytes per GEMM launch from ncu (profiles/gemm_pair_kernel_block_dit_mlp.md)",
                     "kernel": "gemm_pair_kernel<PROMOTE,SWAP> (both GEMMs, CUDA events on the launch stream)",
                     "peak_note": f"dense int8 = 2 x {peak_kind} cuBLAS bf16 burst ({peaks.get('bf16_tflops')} TF/s)",
                     "per_gemm_ms": {"w1_gelu": round(statistics.mean(g1), 4), "w2": round(statistics.mean(g2), 4)}},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": probe.summary(),
    }
    if not args.no_cpu_baseline and world == 1:
        torch.set_num_threads(cpu_cores())
        cv, cmed, sample = run_cpu(args.cpu_tokens, 2, 1)
        line["cpu_baseline"] = {"value": round(cv, 4), "unit": UNIT, "cores": cpu_cores(), "kind": "port",
                                "sample": sample, "s_per_step": round(cmed, 3)}
    print(json.dumps(line), flush=True)
    _finish(world)


def _finish(world):
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def cpu_other_workload(workload: str, steps: int, warmup: int):
    """CPU oracle port of the quip_linear / conversion workloads on a bounded
    sample; returns (metric, unit, value, seconds per sample, sample)."""
    import oracle as O
    from convert_to_quant_quip_int8_b200.workloads import SingleQuipLinear, conversion_sweep_tensors, quip_signs

    if workload == "quip_linear":
        wl = SingleQuipLinear()
        su, sv = (t.numpy() for t in wl.signs())
        qr, sr, _ = O.quip_convert(wl.weight().float().numpy(), su, sv, store_transformed=True)
        x = wl.activations().float().numpy()[:128]
        b = wl.bias().float().numpy()
        step = lambda: O.quip_linear_w8a8(x, qr, sr, su, sv, wl.dim, b)
        unit_ops, scale = 2 * 128 * wl.dim * wl.dim, None
        metric, unit, sample = ("QuIP W8A8 rotated linear TOPS (transformed storage, tensorwise scale)", "TOPS",
                                "128 of 512 tokens through K1 -> int32 GEMM -> K3 (numpy oracle port)")
    else:
        w = (np.random.default_rng(0).standard_normal((3072, 3072)) * 0.02).astype(np.float32)
        su, sv = (t.numpy() for t in quip_signs(1000, 4096, 4096))
        step = lambda: O.quip_convert(O.round_bf16(w), su, sv, "block")
        shapes = [(m, n) for _, m, n in conversion_sweep_tensors()]
        pad = lambda m, n: (1 << (m - 1).bit_length()) * (1 << (n - 1).bit_length())
        scale = sum(pad(m, n) for m, n in shapes) / pad(3072, 3072)  # cost ~ padded elements
        unit_ops = None
        metric, unit, sample = ("QuIP conversion sweep tensors/s (304 tensors, 12.9 B params)", "tensors/s",
                                "one 3072x3072 tensor (padded 4096x4096) through the numpy oracle converter, "
                                "scaled to the sweep by padded element count")
    for _ in range(max(0, warmup)):
        step()
    times = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    value = unit_ops / med / 1e12 if unit_ops else 304 / (med * scale)
    return metric, unit, value, med, sample


def main_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cores = cpu_cores()
    torch.set_num_threads(cores)
    config = {"workload": WORKLOAD, "tokens": 4096, "hidden": 3072, "ffn": 12288, "block": 128,
              "parallelism": "cpu"}
    metric, unit, scaling = METRIC, UNIT, "weak"
    if args.workload in ("flux_stack", "t5_stack"):
        from convert_to_quant_quip_int8_b200.stack import STACKS
        name = args.workload.split("_")[0]
        value, med, sample = run_cpu_stack(name, args.steps, args.warmup)
        metric, unit = f"{name} W8A8 linear-stack tokens/s", "tokens/s"
        config = {"workload": STACKS[name]["describe"], "parallelism": "cpu"}
        scaling = "weak" if args.shard == "replica" else "strong"
    elif args.workload in ("quip_linear", "conversion"):
        metric, unit, value, med, sample = cpu_other_workload(args.workload, args.steps, args.warmup)
        config = {"workload": args.workload, "parallelism": "cpu"}
        scaling = "weak" if args.workload == "quip_linear" else "strong"
    else:
        value, med, sample = run_cpu(args.cpu_tokens, args.steps, args.warmup)
    line = {"impl": "reference", "metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(med * 1e3, 2),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "int8 x int8 -> int32 (fp32 epilogue)", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
