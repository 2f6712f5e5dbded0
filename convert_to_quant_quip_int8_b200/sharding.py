"""Multi-GPU use of the QuIP W8A8 path (one process per GPU).

* Conversion sweep: weight tensors are independent units.  ``plan_partition``
  assigns them to ranks by longest-processing-time on the padded element
  count (the converter's cost); every rank computes the same plan and
  converts its own share -- no collective on the data path.
* Column-sharded linear: rank r holds output rows ``[r*N/G, (r+1)*N/G)`` of the
  int8 weight and its scale slice, computes its ``[T, N/G]`` slice with the
  W8A8 kernels and an NCCL all-gather assembles ``[T, N]`` (every rank gets
  the full output, as a column-parallel linear with gathered output).
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


class ColumnShardedW8A8Linear:
    """Column-parallel W8A8 linear with per-token activation quantization.

    ``weight_q`` ``[N, K]`` int8 and ``scale`` (scalar, ``[N]``/``[N,1]``, or
    ``[N, K/128(,1)]`` block scales) describe the full layer; this rank keeps
    its ``N/G`` rows.  ``N`` must divide by ``16 * G`` (GEMM row alignment).
    """

    def __init__(self, weight_q: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor], rank: int, world: int,
                 group=None, block: int = 128):
        N, K = weight_q.shape
        assert N % (16 * world) == 0, f"N={N} must divide by 16 * world ({world})"
        n_loc = N // world
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
        self.world, self.group = world, group

    def local(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        xq, xs = ops.quant_rows(x2, L.QI8_Q_TOKEN)
        return ops.gemm_i8(xq, self.w, xs, L.QI8_S_ROW, self.s, self.kind, self.bias, x.dtype)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        y = gather_columns(self.local(x), self.world, self.group)
        return y.reshape(*x.shape[:-1], y.shape[-1])
