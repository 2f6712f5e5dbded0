"""Device-resident W8A8 linear stacks (the Flux-shaped transformer and the
T5-XXL encoder), run through the C ABI with preallocated buffers so that a
whole forward can be captured once and replayed as a CUDA graph.

* ``flux``: hidden 3072; 19 double-stream blocks x {img T=4096, txt T=512} x
  {qkv 3072->9216, proj 3072->3072, mlp0 3072->12288, mlp2 12288->3072} and
  38 single-stream blocks (T=4608) x {linear1 3072->21504, linear2
  15360->3072} = 228 linears with bias.  QuIP W8A8 tensorwise weights: the
  two-sided Hadamard conversion with the converter's default per-row requant
  scale ``[N, 1]`` (converters/quip_int8.py:1639-1642), stored in original
  space.
* ``t5``: d_model 4096, d_ff 10240, 24 layers x {q, k, v, o 4096->4096,
  wi_0, wi_1 4096->10240, wo 10240->4096} = 168 linears without bias, batch
  8 x 512 tokens; axis-wise weight scales ``[N]``
  (``AxisWiseINT8Layout``, comfy/quant_ops.py:330-339).

Independent linears overlap: a double block's txt linears (and T5's q, k
and v, wi_0 and wi_1) run on their own streams ("lanes") of the captured
graph, forked at the start of their group and joined at its end, each lane
with its own quantization, workspace and output buffers.  Small per-rank
GEMMs of a token split fill few CTA pairs, so another lane's GEMM runs on
the idle SMs.

Each linear is the reference's W8A8 forward (comfy/quant_ops.py:461-475):
per-token int8 quantization of the bf16 input (K1), then the int8 GEMM with
the fused ``acc * (x_s * w_s) + bias`` epilogue (K2) to bf16.  Inputs are
seeded synthetic activations resident in HBM, one per input shape, except
the Flux MLP down projections, which read GELU(up projection) through K1's
fused GELU.  Attention, norms and modulation are outside the stack.

Multi-GPU (one process per GPU):
* ``replica``: every rank runs the whole stack on its own batch.
* ``tokens``: every rank holds all weights and runs every linear on its 1/G
  of the forward's tokens -- no exchange inside the linear stack.
* ``columns``: every linear is column-sharded -- rank r holds weight rows
  ``[r N/G, (r+1) N/G)`` -- and K1 runs on every rank.  ``gather="peer"``:
  the GEMM epilogue stores each tile into every rank's peer-mapped output
  buffer (``qi8_gemm_i8_gather``) and a peer barrier follows.
  ``gather="nccl"``: the local GEMM runs in token chunks whose NCCL
  all-gathers overlap the next chunk and ``qi8_gather_layout`` assembles
  ``[T, N]`` on every rank.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib as L
from . import ops
from .sharding import PeerWorkspace, token_chunks
from .workloads import flux_linears, gen, next_pow2, student_t_outliers, t5_linears


@dataclass
class LinearSpec:
    name: str
    tokens: int
    k: int
    n: int
    src: str = "x"      # "x": synthetic activation [tokens, k]; otherwise the linear whose output feeds this one
    gelu: bool = False  # GELU of the input, fused into the per-token quantization
    lane: int = 0       # > 0: runs on that lane's stream, concurrently with the other lanes of its group
    group: str = ""     # consecutive specs of one non-empty group fork at its start and join at its end


def flux_specs() -> List[LinearSpec]:
    specs = []
    for name, t, k, n in flux_linears():
        # a double block's txt linears are independent of its img linears
        lane = 1 if ".txt." in name else 0
        group = name.split(".")[0] if name.startswith("double") else ""
        if name.endswith(".mlp2"):
            specs.append(LinearSpec(name, t, k, n, name[: -len("mlp2")] + "mlp0", True, lane, group))
        else:
            specs.append(LinearSpec(name, t, k, n, lane=lane, group=group))
    return specs


def t5_specs() -> List[LinearSpec]:
    # q, k, v read the same input; so do wi_0 and wi_1
    lane = {"k": 1, "v": 2, "wi_1": 1}
    group = {"q": "qkv", "k": "qkv", "v": "qkv", "wi_0": "wi", "wi_1": "wi"}
    specs = []
    for name, t, k, n in t5_linears():
        pre, part = name.split(".")
        g = f"{pre}.{group[part]}" if part in group else ""
        specs.append(LinearSpec(name, t, k, n, lane=lane.get(part, 0), group=g))
    return specs


STACKS = {
    "flux": dict(specs=flux_specs, tokens=4096 + 512, bias=True, quip=True, w_seed=20, x_seed=100,
                 describe="Flux-shaped stack: 19 double blocks (img 4096 + txt 512 tokens) + 38 single blocks "
                          "(4608 tokens), 228 QuIP W8A8 linears, per-row [N,1] scales, bias"),
    "t5": dict(specs=t5_specs, tokens=8 * 512, bias=False, quip=False, w_seed=32, x_seed=30,
               describe="T5-XXL encoder: 24 layers x {q,k,v,o 4096->4096, wi_0/wi_1 4096->10240, "
                        "wo 10240->4096}, 4096 tokens, axis-wise [N] scales"),
}


def fork_groups(specs: List[LinearSpec]) -> List[Tuple[List[int], bool]]:
    """Consecutive specs of one non-empty group form a group; every other
    spec is a group of its own.  Returns (spec indices, forks) per group in
    order, where ``forks`` says whether the group has linears on lanes > 0."""
    groups: List[List[int]] = []
    for i, sp in enumerate(specs):
        if groups and sp.group and specs[i - 1].group == sp.group:
            groups[-1].append(i)
        else:
            groups.append([i])
    return [(ix, any(specs[j].lane for j in ix)) for ix in groups]


def ops_per_forward(specs: List[LinearSpec]) -> int:
    return sum(2 * s.tokens * s.k * s.n for s in specs)


class LinearStack:
    """One stack on one rank: int8 weights (full, or this rank's column
    shard), synthetic inputs and every intermediate buffer, preallocated."""

    def __init__(self, name: str, device: torch.device, rank: int = 0, world: int = 1, shard: str = "replica",
                 chunks: int = 4, group=None, specs: Optional[List[LinearSpec]] = None, gather: str = "peer",
                 overlap: bool = True):
        cfg = STACKS[name]
        self.name, self.cfg, self.device = name, cfg, device
        self.specs = cfg["specs"]() if specs is None else list(specs)
        if shard == "tokens" and world > 1:
            # token split: full weights on every rank, each rank its 1/G of every linear's tokens
            for sp in self.specs:
                assert sp.tokens % world == 0, f"{sp.name}: {sp.tokens} tokens do not split over {world} ranks"
            self.specs = [LinearSpec(sp.name, sp.tokens // world, sp.k, sp.n, sp.src, sp.gelu, sp.lane, sp.group)
                          for sp in self.specs]
        self.rank, self.world, self.group = rank, world, group
        self.sharded = shard == "columns" and world > 1
        # lane streams only where lanes exist and no collective orders the linears
        self.overlap = overlap and not self.sharded and any(sp.lane for sp in self.specs)
        lanes = sorted({sp.lane for sp in self.specs if sp.lane}) if self.overlap else []
        self.sides = {ln: torch.cuda.Stream(device) for ln in lanes}
        self.groups = fork_groups(self.specs) if self.overlap else [([i], False) for i in range(len(self.specs))]
        # per forked group: the fork event, and a join event per lane
        self.fork_events = [(torch.cuda.Event(), {ln: torch.cuda.Event() for ln in self.sides})
                            for ix, f in self.groups if f]
        self.chunks = chunks
        self.gather = gather  # column mode: "peer" (fused into the GEMM epilogue) or "nccl"
        self.peer = None
        self.lib = L.load()
        self._build_weights()
        self._build_buffers()

    # ------------------------------------------------------------ weights
    def _build_weights(self):
        cfg, dev = self.cfg, self.device
        g = torch.Generator(device=dev)
        ws = None
        if cfg["quip"]:
            max_ws = max(ops.quip_workspace_bytes(s.n, s.k) for s in self.specs)
            ws = torch.empty(max_ws, dtype=torch.uint8, device=dev)
        self.weights: List[Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]] = []
        for i, s in enumerate(self.specs):
            g.manual_seed(cfg["w_seed"] + i)
            w = (torch.randn(s.n, s.k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            if cfg["quip"]:
                g.manual_seed(2000 + i)
                su = (torch.randint(0, 2, (next_pow2(s.n),), generator=g, device=dev) * 2 - 1).float()
                sv = (torch.randint(0, 2, (next_pow2(s.k),), generator=g, device=dev) * 2 - 1).float()
                q, sc, _ = ops.quip_convert(w, su, sv, requant=L.QI8_REQ_ROW, want_dequant=False, workspace=ws)
            else:
                q, sc = ops.quant_weight(w, L.QI8_S_ROW)
            del w
            sc = sc.reshape(s.n)
            bias = None
            if cfg["bias"]:
                g.manual_seed(5000 + i)
                bias = (torch.randn(s.n, generator=g, device=dev) * 0.01).to(torch.bfloat16)
            if self.sharded:
                assert s.n % (16 * self.world) == 0, f"{s.name}: N={s.n} does not split over {self.world} ranks"
                n_loc = s.n // self.world
                rows = slice(self.rank * n_loc, (self.rank + 1) * n_loc)
                q, sc = q[rows].contiguous(), sc[rows].contiguous()
                bias = None if bias is None else bias[rows].contiguous()
            self.weights.append((q, sc, bias))
        torch.cuda.synchronize(dev)

    # ------------------------------------------------------------ buffers
    def _build_buffers(self):
        dev, cfg = self.device, self.cfg
        consumed = {s.src for s in self.specs if s.src != "x"}
        self.inputs: Dict[Tuple[int, int], torch.Tensor] = {}
        for s in self.specs:
            key = (s.tokens, s.k)
            if s.src == "x" and key not in self.inputs:
                seed = cfg["x_seed"] + len(self.inputs)
                if self.name == "t5":
                    x = student_t_outliers(torch.randn(s.tokens, s.k, generator=gen(seed)), 0.01, 3, seed + 1)
                    self.inputs[key] = x.to(torch.bfloat16).to(dev)
                else:
                    g = torch.Generator(device=dev)
                    g.manual_seed(seed)
                    self.inputs[key] = torch.randn(s.tokens, s.k, generator=g, device=dev).to(torch.bfloat16)
        max_tn = max(s.tokens * s.n for s in self.specs)
        # per lane: quantized activations, their scales, the split-K
        # workspace (GEMMs whose output tiles fill few CTA pairs split K into
        # exact int32 partial planes reduced by a second pass) and an output
        # scratch; lane 0's are also the attributes xq, xs, ws, scratch
        self.lane_bufs: Dict[int, Dict[str, object]] = {}
        for ln in sorted({self.lane(s) for s in self.specs}):
            mine = [s for s in self.specs if self.lane(s) == ln]
            ws_bytes = 0
            if not self.sharded:
                ws_bytes = max(int(self.lib.qi8_gemm_workspace_bytes(s.tokens, s.n, s.k, L.QI8_S_ROW, L.QI8_S_ROW))
                               for s in mine)
            self.lane_bufs[ln] = {
                "xq": torch.empty(max(s.tokens * s.k for s in mine), dtype=torch.int8, device=dev),
                "xs": torch.empty(max(s.tokens for s in mine), dtype=torch.float32, device=dev),
                "ws": torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev),
                "ws_bytes": ws_bytes,
            }
        b0 = self.lane_bufs[0] if 0 in self.lane_bufs else next(iter(self.lane_bufs.values()))
        self.xq, self.xs, self.ws, self.ws_bytes = b0["xq"], b0["xs"], b0["ws"], b0["ws_bytes"]
        # consumed outputs get their own buffer per (lane, tokens, n); the rest share their lane's scratch
        keys = []
        for s in self.specs:
            key = (self.lane(s), s.tokens, s.n)
            if s.name in consumed and key not in keys:
                keys.append(key)
        if self.sharded and self.gather == "peer":
            # every output lives in a peer-mapped buffer: the scratch is buffer 0, kept outputs follow
            self.peer = PeerWorkspace(max_tn * 2, self.world, self.rank, self.group, 1 + len(keys), dev)
            self.peer_index = {k: 1 + i for i, k in enumerate(keys)}
            self.kept = {k: self.peer.buffer(1 + i, k[1:], torch.bfloat16) for i, k in enumerate(keys)}
            self.lane_bufs[0]["scratch"] = self.peer.bufs[0].view(torch.bfloat16)
        else:
            self.kept = {k: torch.empty(*k[1:], dtype=torch.bfloat16, device=dev) for k in keys}
            for ln, lb in self.lane_bufs.items():
                lb["scratch"] = torch.empty(max(s.tokens * s.n for s in self.specs if self.lane(s) == ln),
                                            dtype=torch.bfloat16, device=dev)
        self.scratch = b0["scratch"]
        self.out_of = {}
        for s in self.specs:
            key = (self.lane(s), s.tokens, s.n)
            buf = self.kept.get(key) if s.name in consumed else None
            scratch = self.lane_bufs[self.lane(s)]["scratch"]
            self.out_of[s.name] = buf if buf is not None else scratch[: s.tokens * s.n].view(s.tokens, s.n)
        self.buf_index = {s.name: (self.peer_index[(0, s.tokens, s.n)] if self.peer is not None and s.name in consumed
                                   else 0) for s in self.specs}
        if self.sharded and self.gather == "nccl":
            max_tnl = max(s.tokens * (s.n // self.world) for s in self.specs)
            self.y_loc = torch.empty(max_tnl, dtype=torch.bfloat16, device=dev)
            self.gathered = torch.empty(max_tn, dtype=torch.bfloat16, device=dev)

    def lane(self, s: LinearSpec) -> int:
        """Stream lane of a linear: its own lane when lanes overlap, else 0."""
        return s.lane if self.overlap else 0

    def source(self, s: LinearSpec) -> torch.Tensor:
        return self.inputs[(s.tokens, s.k)] if s.src == "x" else self.out_of[s.src]

    # ------------------------------------------------------------ forward
    def _k1(self, x: torch.Tensor, s: LinearSpec, sp):
        lb = self.lane_bufs[self.lane(s)]
        mode = L.QI8_Q_TOKEN | (L.QI8_Q_GELU if s.gelu else 0)
        L.check(self.lib.qi8_quant_rows(L.ptr(x), L.QI8_BF16, s.tokens, s.k, s.k, mode, 128, L.ptr(lb["xq"]), s.k,
                                        L.ptr(lb["xs"]), sp), "qi8_quant_rows")

    def _gemm(self, i: int, s: LinearSpec, lo: int, hi: int, out_ptr: int, ld_out: int, sp):
        q, sc, bias = self.weights[i]
        lb = self.lane_bufs[self.lane(s)]
        n = q.shape[0]
        a = lb["xq"].data_ptr() + lo * s.k
        xs = lb["xs"].data_ptr() + lo * 4
        L.check(self.lib.qi8_gemm_i8_ws(ctypes.c_void_p(a), L.ptr(q), hi - lo, n, s.k, ctypes.c_void_p(xs),
                                        L.QI8_S_ROW, L.ptr(sc), L.QI8_S_ROW, L.ptr(bias),
                                        L.QI8_BF16 if bias is not None else 0, ctypes.c_void_p(out_ptr), L.QI8_BF16,
                                        ld_out, L.QI8_ACT_NONE, L.ptr(lb["ws"]), lb["ws_bytes"], sp),
                "qi8_gemm_i8_ws")

    def run_linear(self, i: int, sp, events=None):
        s = self.specs[i]
        self._k1(self.source(s), s, sp)
        out = self.out_of[s.name]
        if events is not None:
            events[0].record()
        if not self.sharded:
            self._gemm(i, s, 0, s.tokens, out.data_ptr(), s.n, sp)
            if events is not None:
                events[1].record()
            return
        n_loc = s.n // self.world
        if self.peer is not None:
            q, sc, bias = self.weights[i]
            xq = self.xq[: s.tokens * s.k].view(s.tokens, s.k)
            L.check(self.lib.qi8_gemm_i8_gather(
                L.ptr(xq), L.ptr(q), s.tokens, n_loc, s.k, L.ptr(self.xs), L.QI8_S_ROW, L.ptr(sc), L.QI8_S_ROW,
                L.ptr(bias), L.QI8_BF16 if bias is not None else 0, self.peer.out_bases(self.buf_index[s.name]),
                self.world, self.rank, L.QI8_BF16, s.n, L.QI8_ACT_NONE, sp), "qi8_gemm_i8_gather")
            if events is not None:
                events[1].record()
            self.peer.barrier(sp)
            return
        y_loc = self.y_loc[: s.tokens * n_loc].view(s.tokens, n_loc)
        gathered = self.gathered[: s.tokens * s.n]
        pending = []
        for lo, hi in token_chunks(s.tokens, self.chunks):
            self._gemm(i, s, lo, hi, y_loc[lo:hi].data_ptr(), n_loc, sp)
            buf = gathered[lo * s.n: hi * s.n].view(self.world * (hi - lo), n_loc)
            pending.append((dist.all_gather_into_tensor(buf, y_loc[lo:hi], group=self.group, async_op=True),
                            buf, lo, hi))
        if events is not None:
            events[1].record()
        for work, buf, lo, hi in pending:
            work.wait()
            L.check(self.lib.qi8_gather_layout(L.ptr(buf), L.QI8_BF16, self.world, hi - lo, n_loc,
                                               ctypes.c_void_p(out[lo:hi].data_ptr()), s.n, sp),
                    "qi8_gather_layout")

    def forward(self, events=None):
        """One forward on the current stream.  With ``events`` (a start/end
        event pair per linear around its GEMM launches) every linear runs on
        the current stream in spec order, so each GEMM is timed alone;
        otherwise each group with linears on lanes > 0 forks them onto their
        lanes' streams and joins them at the group's end (graph-capturable)."""
        sp = L.stream_ptr(self.device)
        if events is not None or not self.overlap:
            for i in range(len(self.specs)):
                self.run_linear(i, sp, None if events is None else events[i])
            return
        main = torch.cuda.current_stream(self.device)
        ptrs = {ln: ctypes.c_void_p(st.cuda_stream) for ln, st in self.sides.items()}
        forks = iter(self.fork_events)
        for ix, forked in self.groups:
            if not forked:
                for i in ix:
                    self.run_linear(i, sp)
                continue
            fork, joins = next(forks)
            used = sorted({self.specs[i].lane for i in ix if self.specs[i].lane})
            fork.record(main)
            for ln in used:
                self.sides[ln].wait_event(fork)
            for i in ix:
                ln = self.specs[i].lane
                self.run_linear(i, ptrs[ln] if ln else sp)
            for ln in used:
                joins[ln].record(self.sides[ln])
                main.wait_event(joins[ln])

    def launches_per_forward(self) -> int:
        """Kernels of this library launched by one forward (K1 + GEMMs + layouts)."""
        if not self.sharded:
            # K1 + GEMM, plus the reduce pass of every GEMM that splits K
            split = sum(1 for s in self.specs
                        if self.lib.qi8_gemm_workspace_bytes(s.tokens, s.n, s.k, L.QI8_S_ROW, L.QI8_S_ROW) > 0)
            return 2 * len(self.specs) + split
        if self.peer is not None:
            return 3 * len(self.specs)  # K1, fused GEMM + gather, peer barrier
        return sum(1 + 2 * len(token_chunks(s.tokens, self.chunks)) for s in self.specs)

    def close(self):
        if self.peer is not None:
            self.peer.close()

    def gemm_ops_local(self) -> int:
        """Multiply-add ops of this rank's GEMMs per forward."""
        return sum(2 * s.tokens * s.k * w[0].shape[0] for s, w in zip(self.specs, self.weights))

    def host_inputs(self) -> Dict[Tuple[int, int], torch.Tensor]:
        return {k: v.cpu().pin_memory() for k, v in self.inputs.items()}
