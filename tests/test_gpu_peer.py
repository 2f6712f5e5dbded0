"""Fused column gather: qi8_gemm_i8_gather writes its tile into every
destination buffer (checked on one GPU with local buffers standing in for
the peers' -- no barrier involved), and on two GPUs the column-parallel
linear over IPC-mapped buffers + peer barrier equals the unsharded layer bit
for bit."""

import ctypes
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import ops, sharding

pytestmark = pytest.mark.gpu


def _gather_call(xq, xs, w, s, kind, bias, bases, world, rank, dtype, N, act=L.QI8_ACT_NONE):
    arr = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bases])
    L.check(L.load().qi8_gemm_i8_gather(L.ptr(xq), L.ptr(w), xq.shape[0], w.shape[0], xq.shape[1], L.ptr(xs),
                                        L.QI8_S_ROW, L.ptr(s), kind, L.ptr(bias),
                                        L.dtype_code(bias.dtype) if bias is not None else 0, arr, world, rank,
                                        L.dtype_code(dtype), N, act, L.stream_ptr()), "qi8_gemm_i8_gather")


@pytest.mark.parametrize("T", [100, 700])
@pytest.mark.parametrize("kind", ["row", "block", "scalar"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("world,rank", [(1, 0), (2, 1), (4, 2)])
def test_gemm_gather_writes_every_destination(T, kind, dtype, world, rank):
    r = np.random.default_rng(T + world)
    K, n_loc = 512, 256
    N = world * n_loc
    x = torch.from_numpy(r.standard_normal((T, K)).astype(np.float32)).to(torch.bfloat16).cuda()
    w = (torch.from_numpy(r.standard_normal((N, K)).astype(np.float32)) * 0.02).cuda()
    req = {"row": L.QI8_REQ_ROW, "block": L.QI8_REQ_BLOCK, "scalar": L.QI8_REQ_GLOBAL}[kind]
    q, s = ops.requant_weight(w, req)
    bias = torch.from_numpy(r.standard_normal(N).astype(np.float32) * 0.1).to(torch.bfloat16).cuda()
    xq, xs = ops.quant_rows(x, L.QI8_Q_TOKEN)
    full = ops.gemm_i8(xq, q, xs, L.QI8_S_ROW, s, None, bias, dtype)
    rows = slice(rank * n_loc, (rank + 1) * n_loc)
    if kind == "scalar":
        s_loc, k_code = s.reshape(()), L.QI8_S_SCALAR
    elif kind == "row":
        s_loc, k_code = s.reshape(N)[rows].contiguous(), L.QI8_S_ROW
    else:
        s_loc, k_code = s.reshape(N, -1)[rows].contiguous(), L.QI8_S_ROW_KBLOCK
    bases = [torch.full((T, N), float("nan"), dtype=dtype, device="cuda") for _ in range(world)]
    _gather_call(xq, xs, q[rows].contiguous(), s_loc, k_code, bias[rows].contiguous(), bases, world, rank, dtype, N)
    torch.cuda.synchronize()
    for b in bases:
        assert torch.equal(b[:, rows], full[:, rows])
        others = torch.cat([b[:, : rank * n_loc], b[:, (rank + 1) * n_loc:]], dim=1)
        assert bool(torch.isnan(others.float()).all())  # nothing written outside this rank's columns


def test_gemm_gather_rejects_bad_arguments():
    xq = torch.zeros(16, 128, dtype=torch.int8, device="cuda")
    xs = torch.ones(16, 1, device="cuda")
    w = torch.zeros(32, 128, dtype=torch.int8, device="cuda")
    s = torch.ones(32, device="cuda")
    out = torch.zeros(16, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(AssertionError):
        _gather_call(xq, xs, w, s, L.QI8_S_ROW, None, [out] * 9, 9, 0, torch.bfloat16, 64)  # > QI8_MAX_PEERS
    with pytest.raises(AssertionError):
        _gather_call(xq, xs, w, s, L.QI8_S_ROW, None, [out, out], 2, 0, torch.bfloat16, 48)  # ld_out < world*n_loc
    with pytest.raises(TypeError):
        _gather_call(xq, xs, w, s, L.QI8_S_ROW, None, [out.int()], 1, 0, torch.int32, 64)


def test_peer_workspace_single_rank():
    ws = sharding.PeerWorkspace(1 << 20, 1, 0, n_buffers=2)
    try:
        for _ in range(3):
            ws.barrier()
        torch.cuda.synchronize()
        ops.device_status()
        assert int(ws.flags[L.QI8_MAX_PEERS].item()) == 3  # completed-barrier counter
        assert ws.next_buffer() == 0 and ws.next_buffer() == 1 and ws.next_buffer() == 0
    finally:
        ws.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    import datetime
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        r = np.random.default_rng(9)
        T, K, N = 777, 1024, 1536
        w = (torch.from_numpy(r.standard_normal((N, K)).astype(np.float32)) * 0.02).cuda()
        bias = torch.from_numpy(r.standard_normal(N).astype(np.float32) * 0.1).to(torch.bfloat16).cuda()
        xs_ = [torch.from_numpy(r.standard_normal((T, K)).astype(np.float32)).to(torch.bfloat16).cuda()
               for _ in range(4)]
        ok = True
        for req in (L.QI8_REQ_ROW, L.QI8_REQ_BLOCK):
            wq, wsc = ops.requant_weight(w, req)
            ref = sharding.ColumnShardedW8A8Linear(wq, wsc, bias, rank=0, world=1)
            ws = sharding.PeerWorkspace(T * N * 2, world, rank, n_buffers=2)
            lin = sharding.ColumnShardedW8A8Linear(wq, wsc, bias, rank=rank, world=world, peer=ws)
            outs = [lin(x).clone() for x in xs_]  # four calls: both buffers reused
            torch.cuda.synchronize()
            ops.device_status()
            ok = ok and all(torch.equal(o, ref(x)) for o, x in zip(outs, xs_))
            ws.close()
        results.put((rank, ok))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        results.put((rank, repr(e)))


def test_peer_barrier_wait_expires_and_reports():
    """The barrier's bounded wait runs out when a peer never arrives: rank 0
    of a two-rank barrier whose rank-1 flag block is a local buffer nothing
    writes.  The kernel gives up after its 2 s limit and returns, the status
    word reports the expiry, the next barrier arrives without waiting, and
    the context stays usable."""
    import time
    ops.device_status(reset=True)
    mine = torch.zeros(L.QI8_MAX_PEERS + 1, dtype=torch.int32, device="cuda")
    absent = torch.zeros(L.QI8_MAX_PEERS + 1, dtype=torch.int32, device="cuda")
    flags = (ctypes.c_void_p * 2)(mine.data_ptr(), absent.data_ptr())
    lib = L.load()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    L.check(lib.qi8_peer_barrier(flags, 2, 0, L.stream_ptr()), "qi8_peer_barrier")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 1.5 < waited < 30.0, f"barrier returned after {waited:.2f} s"
    # this rank's arrival went into slot 0 of both blocks; its completed-barrier count is 1
    assert absent[0].item() == 1 and mine[0].item() == 1 and mine[L.QI8_MAX_PEERS].item() == 1
    # after an expiry later barriers arrive but do not wait
    t0 = time.perf_counter()
    L.check(lib.qi8_peer_barrier(flags, 2, 0, L.stream_ptr()), "qi8_peer_barrier")
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    assert absent[0].item() == 2 and mine[L.QI8_MAX_PEERS].item() == 2
    with pytest.raises(L.QI8Error, match="expired"):
        ops.device_status(reset=True)
    ops.device_status(reset=True)  # the bit was cleared by the read above
    # the context is still usable: a GEMM runs and is correct
    a = torch.ones(64, 128, dtype=torch.int8, device="cuda")
    c = ops.gemm_i8(a, a[:32].contiguous(), out_dtype=torch.int32)
    assert bool((c == 128).all())


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_gather_two_ranks_equals_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rk, v = q.get(timeout=150)
        res[rk] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res == {0: True, 1: True}, res
