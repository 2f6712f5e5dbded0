"""Multi-GPU use of the QuIP W8A8 path (one process per GPU).

* Conversion sweep: weight tensors are independent units.  ``plan_partition``
  assigns them to ranks by longest-processing-time on the padded element
  count (the converter's cost); every rank computes the same plan and
  converts its own share -- no collective on the data path.
* Column-sharded linear: rank r holds output rows ``[r*N/G, (r+1)*N/G)`` of the
  int8 weight and its scale slice, computes its ``[T, N/G]`` slice with the
  W8A8 kernels and an NCCL all-gather assembles ``[T, N]`` (every rank gets
  the full output, as a column-parallel linear with gathered output).  The
  local GEMM runs in token chunks whose all-gathers overlap the next chunk's
  GEMM; ``qi8_gather_layout`` writes each gathered chunk into ``[T, N]``.
  ``qi8_allgather_cols`` offers the same gather through the C ABI for
  callers holding a raw NCCL communicator.
* Fused column gather (``PeerWorkspace`` + ``gemm_gather``): the output
  buffers of all ranks are mapped into every rank (CUDA IPC) and the GEMM
  epilogue stores each tile into all of them over NVLink
  (``qi8_gemm_i8_gather``), followed by a stream-ordered peer barrier -- no
  collective kernel competes with the GEMM for SMs and no re-layout pass
  runs.
"""

from __future__ import annotations

import ctypes
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib as L
from . import ops


def _next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def padded_cost(shape: Tuple[int, int]) -> int:
    return _next_pow2(shape[0]) * _next_pow2(shape[1])


def plan_partition(shapes: Sequence[Tuple[int, int]], world: int) -> List[List[int]]:
    """LPT assignment of tensors (by index) to ``world`` ranks.

    Deterministic: ties are broken by index, so every rank derives the same
    plan without communicating.
    """
    order = sorted(range(len(shapes)), key=lambda i: (-padded_cost(shapes[i]), i))
    loads = [0] * world
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda p: (loads[p], p))
        parts[r].append(i)
        loads[r] += padded_cost(shapes[i])
    return [sorted(p) for p in parts]


def convert_partition(names: Sequence[str], shapes: Sequence[Tuple[int, int]], make_weight: Callable[[int], torch.Tensor],
                      converter, rank: int, world: int, keep: Callable = None) -> Dict[str, tuple]:
    """Convert this rank's share of the tensors; returns ``{name: result}``.

    ``make_weight(i)`` yields tensor ``i`` (on any device); ``keep(result)``
    may reduce what is retained per tensor (e.g. move it to the host).
    """
    out = {}
    for i in plan_partition(shapes, world)[rank]:
        res = converter.convert(make_weight(i))
        out[names[i]] = keep(res) if keep is not None else res
    return out


def cuda_layout(gathered: torch.Tensor, world: int, out: torch.Tensor) -> torch.Tensor:
    """``[world * T, n_loc]`` all-gather result -> ``out [T, world * n_loc]``
    (a row-strided view) with the ``qi8_gather_layout`` kernel."""
    return ops.gather_layout(gathered, world, out=out)


def gather_columns(y_local: torch.Tensor, world: int, group=None, out: Optional[torch.Tensor] = None,
                   layout: Callable = cuda_layout) -> torch.Tensor:
    """All-gather column shards ``[T, N/G]`` of every rank into ``[T, N]``."""
    if world == 1:
        return y_local
    T, n_loc = y_local.shape
    buf = torch.empty((world * T, n_loc), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    if out is None:
        out = torch.empty((T, world * n_loc), dtype=y_local.dtype, device=y_local.device)
    layout(buf, world, out)
    return out


def token_chunks(T: int, chunks: int, unit: int = 256) -> List[Tuple[int, int]]:
    """Splits ``T`` tokens into at most ``chunks`` contiguous ranges whose
    bounds are multiples of ``unit`` (the GEMM's row tile) where possible."""
    units = (T + unit - 1) // unit
    chunks = max(1, min(chunks, units))
    bounds, lo = [], 0
    for c in range(chunks):
        n = units // chunks + (1 if c < units % chunks else 0)
        hi = min(T, lo + n * unit)
        bounds.append((lo, hi))
        lo = hi
    return bounds


def gather_rows_overlapped(produce: Callable[[int, int], torch.Tensor], T: int, chunks: int, world: int,
                           group=None, out: Optional[torch.Tensor] = None,
                           layout: Callable = cuda_layout, unit: int = 256) -> torch.Tensor:
    """Column all-gather overlapped with the producer of the local shard.

    ``produce(lo, hi)`` returns tokens ``lo:hi`` ``[hi - lo, n_loc]`` of the
    local column shard (one GEMM over a row slice of the quantized
    activations, launched on the current stream).  Each chunk's all-gather
    is issued asynchronously -- NCCL runs it on its own stream once the
    chunk's GEMM is done -- so chunk k's transfer overlaps the GEMM of chunk
    k+1; ``layout`` then writes every gathered chunk ``[G, hi-lo, n_loc]``
    into rows ``lo:hi`` of ``out [T, G * n_loc]``.  Every rank issues the same
    collectives in the same order.
    """
    pending = []
    for lo, hi in token_chunks(T, chunks, unit):
        yk = produce(lo, hi).contiguous()
        buf = torch.empty((world * (hi - lo), yk.shape[1]), dtype=yk.dtype, device=yk.device)
        pending.append((dist.all_gather_into_tensor(buf, yk, group=group, async_op=True), buf, lo, hi))
    n_loc = pending[0][1].shape[1]
    if out is None:
        out = torch.empty((T, world * n_loc), dtype=pending[0][1].dtype, device=pending[0][1].device)
    for work, buf, lo, hi in pending:
        work.wait()
        layout(buf, world, out[lo:hi])
    return out


class PeerWorkspace:
    """Peer-mapped output buffers and barrier flags of the fused column gather.

    Every rank allocates ``n_buffers`` buffers of ``nbytes`` and one block of
    ``QI8_MAX_PEERS + 1`` flag words, exports them as CUDA IPC handles
    (``qi8_ipc_handle``), exchanges the handles over ``group`` and maps every
    peer's (``qi8_ipc_open``).  ``out_bases(j)`` is the per-rank pointer array
    of buffer ``j`` for ``qi8_gemm_i8_gather``; ``barrier()`` enqueues
    ``qi8_peer_barrier`` on the current stream.  Collective: every rank
    constructs it (and calls ``close``) in the same order.
    """

    def __init__(self, nbytes: int, world: int, rank: int, group=None, n_buffers: int = 2, device=None):
        assert 1 <= world <= L.QI8_MAX_PEERS, f"at most {L.QI8_MAX_PEERS} ranks"
        self.lib = L.load()
        self.world, self.rank, self.group = world, rank, group
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.bufs = [torch.empty(int(nbytes), dtype=torch.uint8, device=self.device) for _ in range(n_buffers)]
        self.flags = torch.zeros(L.QI8_MAX_PEERS + 1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        local = self.bufs + [self.flags]
        mine = []
        for t in local:
            h = ctypes.create_string_buffer(64)
            off = ctypes.c_int64()
            L.check(self.lib.qi8_ipc_handle(L.ptr(t), h, ctypes.byref(off)), "qi8_ipc_handle")
            mine.append((h.raw, off.value))
        everyone = [None] * world
        if world > 1:
            dist.all_gather_object(everyone, mine, group=group)
        else:
            everyone = [mine]
        # several buffers can sit in one allocation (one IPC handle): map each allocation once
        self._opened = {}
        table = [[0] * world for _ in local]
        for r in range(world):
            for j, (h, off) in enumerate(everyone[r]):
                if r == rank:
                    table[j][r] = local[j].data_ptr()
                    continue
                if (r, h) not in self._opened:
                    base = ctypes.c_void_p()
                    L.check(self.lib.qi8_ipc_open(h, 0, ctypes.byref(base)), "qi8_ipc_open")
                    self._opened[(r, h)] = base.value
                table[j][r] = self._opened[(r, h)] + off
        self._arrays = [(ctypes.c_void_p * world)(*row) for row in table]
        self._next = 0
        if world > 1:
            dist.barrier(group=group)

    def buffer(self, j: int, shape, dtype) -> torch.Tensor:
        n = 1
        for d in shape:
            n *= d
        es = torch.empty((), dtype=dtype).element_size()
        assert n * es <= self.bufs[j].numel(), "peer buffer too small"
        return self.bufs[j][: n * es].view(dtype).view(*shape)

    def out_bases(self, j: int):
        return self._arrays[j]

    def next_buffer(self) -> int:
        """Alternates between the buffers.  With one rank an output stays
        valid until the call after next.  With several ranks it is valid only
        until the next call on this workspace is enqueued: once this rank's
        next peer barrier completes, a peer may start the call after next and
        store into the buffer again, so any read of an output must be enqueued
        on this rank's stream before its next call."""
        j = self._next
        self._next = (self._next + 1) % len(self.bufs)
        return j

    def barrier(self, stream=None):
        sp = L.stream_ptr(self.device) if stream is None else stream
        L.check(self.lib.qi8_peer_barrier(self._arrays[-1], self.world, self.rank, sp), "qi8_peer_barrier")

    def close(self):
        """Unmaps the peers' buffers (collective; call before freeing)."""
        torch.cuda.synchronize(self.device)
        for base in self._opened.values():
            L.check(self.lib.qi8_ipc_close(ctypes.c_void_p(base), 0), "qi8_ipc_close")
        self._opened = {}
        if self.world > 1:
            dist.barrier(group=self.group)


def gemm_gather(xq: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, s: torch.Tensor, kind: int,
                bias: Optional[torch.Tensor], ws: PeerWorkspace, j: int, N: int, out_dtype: torch.dtype,
                act: int = L.QI8_ACT_NONE) -> torch.Tensor:
    """Column-parallel GEMM whose epilogue writes this rank's tile into
    buffer ``j`` of every rank (``qi8_gemm_i8_gather``), then the peer
    barrier; returns the gathered ``[T, N]`` view of the local buffer."""
    T, K = xq.shape
    n_loc = w.shape[0]
    out = ws.buffer(j, (T, N), out_dtype)
    L.check(ws.lib.qi8_gemm_i8_gather(L.ptr(xq), L.ptr(w), T, n_loc, K, L.ptr(xs), L.QI8_S_ROW, L.ptr(s), kind,
                                      L.ptr(bias), L.dtype_code(bias.dtype) if bias is not None else 0,
                                      ws.out_bases(j), ws.world, ws.rank, L.dtype_code(out_dtype), N, act,
                                      L.stream_ptr(xq.device)), "qi8_gemm_i8_gather")
    ws.barrier()
    return out


class ColumnShardedW8A8Linear:
    """Column-parallel W8A8 linear with per-token activation quantization.

    ``weight_q`` ``[N, K]`` int8 and ``scale`` (scalar, ``[N]``/``[N,1]``, or
    ``[N, K/128(,1)]`` block scales) describe the full layer; this rank keeps
    its ``N/G`` rows (``N`` must divide by ``16 * G``).  With ``G > 1`` the
    local GEMM runs in ``chunks`` token ranges whose all-gathers overlap the
    next range's GEMM (``chunks`` defaults to 4 when ``G > 1``).
    """

    def __init__(self, weight_q: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor], rank: int, world: int,
                 group=None, block: int = 128, chunks: Optional[int] = None,
                 peer: Optional[PeerWorkspace] = None):
        N, K = weight_q.shape
        assert N % (16 * world) == 0, f"N={N} must divide by 16 * world ({world})"
        n_loc = N // world
        rows = slice(rank * n_loc, (rank + 1) * n_loc)
        if scale.numel() == 1:
            s_loc = scale.reshape(())
        elif scale.numel() == N:
            s_loc = scale.reshape(N)[rows]
        else:
            assert scale.numel() == N * (K // block), f"scale of shape {tuple(scale.shape)}"
            s_loc = scale.reshape(N, -1)[rows]
        self._init_local(weight_q[rows], s_loc, None if bias is None else bias[rows], world, group, block, chunks,
                         peer)

    @classmethod
    def from_local(cls, weight_shard: torch.Tensor, scale_shard: torch.Tensor, bias_shard: Optional[torch.Tensor],
                   world: int, group=None, block: int = 128, chunks: Optional[int] = None,
                   peer: Optional[PeerWorkspace] = None):
        """Builds the layer from this rank's rows ``[N/G, K]`` of the weight
        and the matching scale / bias slices (a scalar scale is shared)."""
        self = cls.__new__(cls)
        self._init_local(weight_shard, scale_shard, bias_shard, world, group, block, chunks, peer)
        return self

    def _init_local(self, w, s, bias, world, group, block, chunks, peer):
        self.peer = peer
        n_loc, K = w.shape
        assert n_loc % 16 == 0, f"local rows {n_loc} must be a multiple of 16"
        self.w = w.contiguous()
        if s.numel() == 1:
            self.s, self.kind = s.reshape(()).to(torch.float32), L.QI8_S_SCALAR
        elif s.numel() == n_loc:
            self.s, self.kind = s.reshape(n_loc).to(torch.float32).contiguous(), L.QI8_S_ROW
        else:
            assert s.numel() == n_loc * (K // block), f"scale of shape {tuple(s.shape)}"
            self.s, self.kind = s.reshape(n_loc, -1).to(torch.float32).contiguous(), L.QI8_S_ROW_KBLOCK
        self.bias = None if bias is None else bias.contiguous()
        self.world, self.group, self.n_loc = world, group, n_loc
        self.chunks = (4 if world > 1 else 1) if chunks is None else max(1, int(chunks))

    def _gemm(self, xq, xs, out_dtype):
        return ops.gemm_i8(xq, self.w, xs, L.QI8_S_ROW, self.s, self.kind, self.bias, out_dtype)

    def local(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        xq, xs = ops.quant_rows(x2, L.QI8_Q_TOKEN)
        return self._gemm(xq, xs, x.dtype)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        T = x2.shape[0]
        xq, xs = ops.quant_rows(x2, L.QI8_Q_TOKEN)
        if self.peer is not None:
            # fused gather: the output is a view of a peer buffer; with several ranks it is valid only
            # until the next call on this workspace is enqueued (see PeerWorkspace.next_buffer)
            y = gemm_gather(xq, xs, self.w, self.s, self.kind, self.bias, self.peer, self.peer.next_buffer(),
                            self.n_loc * self.world, x.dtype)
        elif self.chunks == 1:
            y = gather_columns(self._gemm(xq, xs, x.dtype), self.world, self.group)
        else:
            y = gather_rows_overlapped(lambda lo, hi: self._gemm(xq[lo:hi], xs[lo:hi], x.dtype), T, self.chunks,
                                       self.world, self.group)
        return y.reshape(*x.shape[:-1], y.shape[-1])
