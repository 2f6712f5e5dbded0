"""qi8_allgather_cols (column all-gather of a column-sharded linear) over a
caller-created NCCL communicator.  One rank on one GPU always; two ranks in
two processes when the box has two GPUs."""

import ctypes
import multiprocessing as mp
import os

import numpy as np
import pytest
import torch

from convert_to_quant_quip_int8_b200 import ops

pytestmark = pytest.mark.gpu


class _UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_char * 128)]  # ncclUniqueId, passed by value


def _libnccl():
    import nvidia.nccl
    path = os.path.join(list(nvidia.nccl.__path__)[0], "lib", "libnccl.so.2")
    lib = ctypes.CDLL(path if os.path.exists(path) else "libnccl.so.2")
    lib.ncclCommInitAll.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    lib.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _UniqueId, ctypes.c_int]
    lib.ncclGetUniqueId.argtypes = [ctypes.POINTER(_UniqueId)]
    lib.ncclCommDestroy.argtypes = [ctypes.c_void_p]
    return lib


def _shard(rank, T, n_loc, dtype):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(T, n_loc, generator=g).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.int32])
def test_allgather_cols_single_rank(dtype):
    torch.cuda.set_device(0)
    nccl = _libnccl()
    comm = ctypes.c_void_p()
    dev = (ctypes.c_int * 1)(0)
    assert nccl.ncclCommInitAll(ctypes.byref(comm), 1, dev) == 0
    try:
        y = _shard(0, 37, 24, dtype).cuda()
        out = ops.allgather_cols(y, comm.value, 1)
        torch.cuda.synchronize()
        assert torch.equal(out.cpu(), y.cpu())
    finally:
        nccl.ncclCommDestroy(comm)


def _rank_main(rank, world, uid, q):
    try:
        torch.cuda.set_device(rank)
        nccl = _libnccl()
        comm = ctypes.c_void_p()
        uid_s = _UniqueId.from_buffer_copy(uid)
        rc = nccl.ncclCommInitRank(ctypes.byref(comm), world, uid_s, rank)
        if rc != 0:
            q.put((rank, f"ncclCommInitRank {rc}"))
            return
        T, n_loc = 33, 48
        y = _shard(rank, T, n_loc, torch.bfloat16).cuda()
        out = ops.allgather_cols(y, comm.value, world)
        torch.cuda.synchronize()
        expect = torch.cat([_shard(r, T, n_loc, torch.bfloat16) for r in range(world)], dim=1)
        q.put((rank, bool(torch.equal(out.cpu(), expect))))
        nccl.ncclCommDestroy(comm)
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_allgather_cols_two_ranks():
    nccl = _libnccl()
    uid = _UniqueId()
    assert nccl.ncclGetUniqueId(ctypes.byref(uid)) == 0
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, bytes(uid), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, v = q.get(timeout=120)
        res[r] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res == {0: True, 1: True}, res
