"""Multi-GPU use of the QuIP W8A8 path (one process per GPU).

* Conversion sweep: weight tensors are independent units.  ``plan_partition``
  assigns them to ranks by longest-processing-time on the padded element
  count (the converter's cost); every rank computes the same plan and
  converts its own share -- no collective on the data path.
* Column-sharded linear: rank r holds output rows ``[r*N/G, (r+1)*N/G)`` of the
  int8 weight and its scale slice, computes its ``[T, N/G]`` slice with the
  W8A8 kernels and an NCCL all-gather assembles ``[T, N]`` (every rank gets
  the full output, as a column-parallel linear with gathered output).  The
  local GEMM runs in column chunks whose all-gathers overlap the next chunk.
  ``qi8_allgather_cols`` offers the same gather through the C ABI for
  callers holding a raw NCCL communicator.
"""

from __future__ import annotations

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


def gather_columns(y_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather column shards ``[T, N/G]`` of every rank into ``[T, N]``."""
    if world == 1:
        return y_local
    T, n_loc = y_local.shape
    buf = torch.empty((world * T, n_loc), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    return buf.view(world, T, n_loc).permute(1, 0, 2).reshape(T, world * n_loc)


def assemble_chunks(gathered: Sequence[torch.Tensor], world: int, T: int) -> torch.Tensor:
    """``[T, N]`` from per-chunk all-gather results.

    Chunk k of rank r holds output columns ``r*n_loc + k*n_c .. +n_c`` (``n_loc =
    len(gathered) * n_c``); ``gathered[k]`` is ``[world*T, n_c]`` in rank order.
    """
    S = len(gathered)
    n_c = gathered[0].shape[1]
    g = torch.stack(list(gathered)).view(S, world, T, n_c)
    return g.permute(2, 1, 0, 3).reshape(T, world * S * n_c)


def gather_columns_overlapped(produce: Callable[[int], torch.Tensor], chunks: int, world: int,
                              group=None) -> torch.Tensor:
    """Column all-gather overlapped with the producer of the local shard.

    ``produce(k)`` returns chunk ``k`` ``[T, n_c]`` of the local shard (e.g. one
    GEMM over a slice of the weight rows, launched on the current stream);
    its all-gather is issued asynchronously (NCCL runs it on its own stream
    after the chunk's producer), so chunk k's transfer overlaps the
    computation of chunk k+1.  Every rank issues the same collectives in the
    same order.
    """
    works, gathered = [], []
    T = None
    for k in range(chunks):
        yk = produce(k).contiguous()
        T = yk.shape[0]
        buf = torch.empty((world * T, yk.shape[1]), dtype=yk.dtype, device=yk.device)
        works.append(dist.all_gather_into_tensor(buf, yk, group=group, async_op=True))
        gathered.append(buf)
    for w in works:
        w.wait()
    return assemble_chunks(gathered, world, T)


class ColumnShardedW8A8Linear:
    """Column-parallel W8A8 linear with per-token activation quantization.

    ``weight_q`` ``[N, K]`` int8 and ``scale`` (scalar, ``[N]``/``[N,1]``, or
    ``[N, K/128(,1)]`` block scales) describe the full layer; this rank keeps
    its ``N/G`` rows.  ``N`` must divide by ``16 * G * chunks`` (GEMM row
    alignment per chunk).  With ``G > 1`` the local GEMM runs in ``chunks``
    column slices whose all-gathers overlap the next slice's GEMM.
    """

    def __init__(self, weight_q: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor], rank: int, world: int,
                 group=None, block: int = 128, chunks: Optional[int] = None):
        N, K = weight_q.shape
        assert N % (16 * world) == 0, f"N={N} must divide by 16 * world ({world})"
        n_loc = N // world
        if chunks is None:
            chunks = 4 if world > 1 else 1
        while chunks > 1 and n_loc % (16 * chunks) != 0:
            chunks //= 2
        self.chunks = chunks
        rows = slice(rank * n_loc, (rank + 1) * n_loc)
        self.w = weight_q[rows].contiguous()
        if scale.numel() == 1:
            self.s, self.kind = scale.reshape(()).to(torch.float32), L.QI8_S_SCALAR
        elif scale.numel() == N:
            self.s, self.kind = scale.reshape(N)[rows].to(torch.float32).contiguous(), L.QI8_S_ROW
        else:
            assert scale.numel() == N * (K // block), f"scale of shape {tuple(scale.shape)}"
            self.s, self.kind = scale.reshape(N, -1)[rows].to(torch.float32).contiguous(), L.QI8_S_ROW_KBLOCK
        self.bias = None if bias is None else bias[rows].contiguous()
        self.world, self.group, self.n_loc = world, group, n_loc

    def _gemm(self, xq, xs, lo, hi, out_dtype):
        s = self.s if self.kind == L.QI8_S_SCALAR else self.s[lo:hi]
        b = None if self.bias is None else self.bias[lo:hi]
        return ops.gemm_i8(xq, self.w[lo:hi], xs, L.QI8_S_ROW, s, self.kind, b, out_dtype)

    def local(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        xq, xs = ops.quant_rows(x2, L.QI8_Q_TOKEN)
        return self._gemm(xq, xs, 0, self.n_loc, x.dtype)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.chunks == 1:
            y = gather_columns(self.local(x), self.world, self.group)
        else:
            x2 = x.reshape(-1, x.shape[-1])
            xq, xs = ops.quant_rows(x2, L.QI8_Q_TOKEN)
            n_c = self.n_loc // self.chunks
            y = gather_columns_overlapped(lambda k: self._gemm(xq, xs, k * n_c, (k + 1) * n_c, x.dtype),
                                          self.chunks, self.world, self.group)
        return y.reshape(*x.shape[:-1], y.shape[-1])
