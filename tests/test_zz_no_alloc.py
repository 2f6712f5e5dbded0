"""The QuIP converter entry point that allocates nothing.

``qi8_quip_convert_noalloc`` serves callers that cannot allocate device
memory (a C-ABI caller without a CUDA allocator of its own, or a process whose
memory sits in another allocator's pool): it runs the same conversion as
``qi8_quip_convert`` on a fixed scratch array inside the library.  These
tests call both entry points through the C ABI and require identical
results on two calls in a row -- the second one smaller than the first, so
stale scratch contents from the first call would show.  The file is named to
be collected last.
"""

import numpy as np
import pytest
import torch

from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import ops

pytestmark = pytest.mark.gpu


def _inputs(M, N, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(M, N, generator=g) * 0.02).to(torch.bfloat16).cuda()
    mp, np_ = 1 << (M - 1).bit_length(), 1 << (N - 1).bit_length()
    su = (torch.randint(0, 2, (mp,), generator=g).float() * 2 - 1).cuda()
    sv = (torch.randint(0, 2, (np_,), generator=g).float() * 2 - 1).cuda()
    return w, su, sv


def _outputs(M, N, requant, block=128):
    dev = torch.device("cuda")
    q = torch.empty((M, N), dtype=torch.int8, device=dev)
    if requant == L.QI8_REQ_BLOCK and N % block == 0:
        s = torch.empty((M, N // block), dtype=torch.float32, device=dev)
    elif requant == L.QI8_REQ_GLOBAL:
        s = torch.empty((1,), dtype=torch.float32, device=dev)
    else:
        s = torch.empty((M,), dtype=torch.float32, device=dev)
    d = torch.empty((M, N), dtype=torch.float32, device=dev)
    return q, s, d


def _call(noalloc, w, su, sv, requant, block=128):
    lib = L.load()
    M, N = w.shape
    q, s, d = _outputs(M, N, requant, block)
    args = [L.ptr(w), L.QI8_BF16, M, N, L.ptr(su), L.ptr(sv), 0, requant, block, L.ptr(q), L.ptr(s), L.ptr(d)]
    if noalloc:
        rc = lib.qi8_quip_convert_noalloc(*args, L.stream_ptr())
    else:
        ws = torch.empty(ops.quip_workspace_bytes(M, N), dtype=torch.uint8, device="cuda")
        rc = lib.qi8_quip_convert(*args, L.ptr(ws), ws.numel(), L.stream_ptr())
    L.check(rc, "quip convert")
    torch.cuda.synchronize()
    return q.cpu().numpy(), s.cpu().numpy(), d.cpu().numpy()


def test_noalloc_matches_workspace_entry_point_twice():
    cases = [((3000, 2048), L.QI8_REQ_BLOCK, 11), ((700, 1000), L.QI8_REQ_GLOBAL, 12)]
    for (M, N), req, seed in cases:
        w, su, sv = _inputs(M, N, seed)
        ref = _call(False, w, su, sv, req)
        got = _call(True, w, su, sv, req)
        for a, b in zip(ref, got):
            assert np.array_equal(a, b)
    L.check(L.load().qi8_device_status(1), "device status")


def test_noalloc_rejects_oversize():
    lib = L.load()
    # 4097 x 4096 pads to 8192 x 4096 = 2^25 elements > the 2^24 built-in scratch
    rc = lib.qi8_quip_convert_noalloc(None, L.QI8_BF16, 4097, 4096, None, None, 0, 0, 128, None, None, None,
                                      L.stream_ptr())
    assert rc == L.QI8_ESHAPE and "exceeds the built-in scratch" in L.last_error()
