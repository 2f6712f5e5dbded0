"""Multi-rank host logic on CPU (gloo): partition plan, column all-gather
layout, and failure propagation when a rank dies before a collective."""

import multiprocessing as mp
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist

from convert_to_quant_quip_int8_b200 import sharding
from convert_to_quant_quip_int8_b200.workloads import conversion_sweep_tensors


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=20):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _torch_layout(gathered, world, out):
    """CPU statement of qi8_gather_layout: [G*T, n] -> out[t, r*n + j] = gathered[r*T + t, j]."""
    T = out.shape[0]
    out.copy_(gathered.view(world, T, -1).permute(1, 0, 2).reshape(T, -1))
    return out


def _worker_plan(rank, world, port, q):
    try:
        _init(rank, world, port)
        tensors = conversion_sweep_tensors()
        shapes = [(m, n) for _, m, n in tensors]
        mine = sharding.plan_partition(shapes, world)[rank]
        everyone = [None] * world
        dist.all_gather_object(everyone, mine)
        # column all-gather layout: rank r contributes columns r*4 .. r*4+3
        T = 3
        y_local = torch.arange(T * 4, dtype=torch.float32).reshape(T, 4) + 100 * rank
        y = sharding.gather_columns(y_local, world, layout=_torch_layout)
        # overlapped gather in token chunks (unit 1 token here): chunk = rows lo:hi of the shard
        chunks = sharding.token_chunks(T, 2, unit=1)
        assert chunks == [(0, 2), (2, 3)]
        y_chunked = sharding.gather_rows_overlapped(lambda lo, hi: y_local[lo:hi], T, 2, world,
                                                    layout=_torch_layout, unit=1)
        q.put((rank, everyone, y, y_chunked))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, "error", repr(e)))


def _worker_fail(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            raise RuntimeError("injected failure before the collective")
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put((rank, "completed"))
    except Exception as e:
        q.put((rank, "error", type(e).__name__))


def _run(target, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 90
    while len(results) < world and time.time() < deadline:
        try:
            item = q.get(timeout=max(0.1, deadline - time.time()))
        except Exception:
            break
        results[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


def test_plan_partition_balanced_and_deterministic():
    tensors = conversion_sweep_tensors()
    assert len(tensors) == 304
    assert sum(m * n for _, m, n in tensors) == 12_910_067_712
    shapes = [(m, n) for _, m, n in tensors]
    for world in (1, 2, 4, 8):
        parts = sharding.plan_partition(shapes, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(shapes)))
        loads = [sum(sharding.padded_cost(shapes[i]) for i in p) for p in parts]
        assert max(loads) / (sum(loads) / world) < 1.02
        assert parts == sharding.plan_partition(shapes, world)


@pytest.mark.parametrize("world", [2])
def test_gloo_plan_agreement_and_column_gather(world):
    res = _run(_worker_plan, world)
    assert len(res) == world, res
    plans = [res[r][0] for r in range(world)]
    assert all(p != "error" for p in plans), res
    assert plans[0] == plans[1]
    assert sorted(i for part in plans[0] for i in part) == list(range(304))
    expect = torch.cat([torch.arange(12, dtype=torch.float32).reshape(3, 4) + 100 * r for r in range(world)], dim=1)
    for r in range(world):
        assert torch.equal(res[r][1], expect)
        assert torch.equal(res[r][2], expect)


def test_gloo_rank_failure_is_reported_not_hung():
    t0 = time.time()
    res = _run(_worker_fail, 2)
    assert res.get(1) == ("error", "RuntimeError")
    assert res.get(0, ("missing",))[0] == "error"  # the survivor's collective fails instead of hanging
    assert time.time() - t0 < 80
