"""One rank's share of a token-split linear stack, timed on one GPU.

With the token split (``bench.py --gpus N``, the default at N > 1) a rank
holds all weights and runs every linear on 1/N of the tokens; nothing is
exchanged inside the stack, so rank 0's forward on one GPU takes the same
device time as on an N-GPU box (the box adds only the barrier and the
max over ranks).  This tool builds rank 0 of an N-way split and times its
forward as a replayed CUDA graph (CUDA events, ``--steps`` replays after
warm-up), plus the GEMM time of one eager forward.  It reports a per-rank
time, not a scaling measurement.

    python benchmarks/stack_rank.py --world 8 [--workload flux|t5] [--steps 20]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from convert_to_quant_quip_int8_b200 import ops  # noqa: E402
from convert_to_quant_quip_int8_b200.stack import STACKS, LinearStack  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--world", type=int, nargs="+", default=[1, 2, 4, 8])
    ap.add_argument("--workload", default="flux", choices=sorted(STACKS))
    ap.add_argument("--steps", type=int, default=20)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    res = {}
    for world in args.world:
        st = LinearStack(args.workload, dev, 0, world, "tokens" if world > 1 else "replica")
        for _ in range(2):
            st.forward()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            st.forward()
        for _ in range(3):
            g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(args.steps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in st.specs]
        st.forward(evs)
        torch.cuda.synchronize()
        gemm_ms = sum(x.elapsed_time(y) for x, y in evs)
        ops.device_status()
        tokens = STACKS[args.workload]["tokens"]
        # GEMM time (incl. a split-K reduce) per distinct (tokens, in, out) shape
        shapes = {}
        for sp, (x, y) in zip(st.specs, evs):
            key = f"{sp.tokens}x{sp.k}x{sp.n}"
            d = shapes.setdefault(key, {"count": 0, "ms": 0.0})
            d["count"] += 1
            d["ms"] += x.elapsed_time(y)
        for key, d in shapes.items():
            t, k, n = (int(v) for v in key.split("x"))
            d["us_each"] = round(d["ms"] * 1e3 / d["count"], 2)
            d["tops"] = round(2 * t * k * n / (d["us_each"] * 1e-6) / 1e12, 1)
            d["ms"] = round(d["ms"], 3)
        res[f"world{world}"] = {"rank_ms_per_forward": round(ms, 3), "gemm_ms_eager": round(gemm_ms, 3),
                                "job_tokens_per_s_if_ranks_match": round(tokens / (ms / 1e3), 1),
                                "launches_per_forward": st.launches_per_forward(), "gemm_by_shape": shapes}
        del g
        st.close()
        del st
        torch.cuda.empty_cache()
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
