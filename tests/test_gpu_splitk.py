"""Split-K of plain-scale GEMMs with few output tiles (qi8_gemm_i8_ws): the
int32 partial planes sum exactly, so every output equals the unsplit GEMM's
bit for bit, and the int32 result equals the oracle's int_mm."""

import numpy as np
import pytest
import torch

import oracle as O
from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import ops

pytestmark = pytest.mark.gpu


def _unsplit(a, b, a_s, a_kind, b_s, b_kind, bias, dtype, act):
    M, K = a.shape
    N = b.shape[0]
    out = torch.empty((M, N), dtype=dtype, device="cuda")
    L.check(L.load().qi8_gemm_i8(L.ptr(a), L.ptr(b), M, N, K, L.ptr(a_s), a_kind, L.ptr(b_s), b_kind, L.ptr(bias),
                                 L.dtype_code(bias.dtype) if bias is not None else 0, L.ptr(out), L.dtype_code(dtype),
                                 N, act, L.stream_ptr()), "qi8_gemm_i8")
    return out


@pytest.mark.parametrize("M,N,K", [(512, 4096, 8192), (300, 512, 8192), (129, 1024, 8192),
                                   # rows <= 128 take the CTA-pair kernel when they split (zero-filled rows)
                                   (64, 3072, 12288), (37, 1024, 9216), (1, 512, 8192),
                                   # a last split shorter than the others, its last K block partial
                                   (200, 1024, 8208),
                                   # per-rank shapes of the Flux stack split over 8 GPUs
                                   (576, 3072, 15360), (512, 3072, 12288)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("kind", ["row", "scalar"])
def test_split_k_equals_unsplit(M, N, K, dtype, kind):
    assert ops._gemm_ws_bytes(M, N, K, L.QI8_S_ROW, L.QI8_S_ROW) > 0, "shape expected to split"
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8).cuda()
    b = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8).cuda()
    a_s = (torch.rand(M, 1, generator=g) * 0.01).cuda()
    if kind == "row":
        b_s, b_kind = (torch.rand(N, generator=g) * 0.01).cuda(), L.QI8_S_ROW
    else:
        b_s, b_kind = torch.tensor(0.003).cuda(), L.QI8_S_SCALAR
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16).cuda()
    for act in (L.QI8_ACT_NONE, L.QI8_ACT_GELU):
        got = ops.gemm_i8(a, b, a_s, L.QI8_S_ROW, b_s, b_kind, bias, dtype, act)
        ref = _unsplit(a, b, a_s, L.QI8_S_ROW, b_s, b_kind, bias, dtype, act)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)


def test_split_k_int32_equals_oracle():
    M, N, K = 512, 2048, 8192
    r = np.random.default_rng(5)
    a = r.integers(-128, 128, (M, K), dtype=np.int8)
    b = r.integers(-128, 128, (N, K), dtype=np.int8)
    assert ops._gemm_ws_bytes(M, N, K, L.QI8_S_NONE, L.QI8_S_NONE) > 0
    got = ops.gemm_i8(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), out_dtype=torch.int32)
    assert np.array_equal(got.cpu().numpy(), O.int_mm(a, b))


def test_split_decision_by_grid_and_scales():
    assert ops._gemm_ws_bytes(4096, 12288, 3072, L.QI8_S_ROW, L.QI8_S_ROW) == 0
    assert ops._gemm_ws_bytes(512, 4096, 4096, L.QI8_S_ROW, L.QI8_S_ROW_KBLOCK) == 0
    # few rows, few tiles: splits only when K is long enough to pay for the reduce
    assert ops._gemm_ws_bytes(64, 4096, 4096, L.QI8_S_ROW, L.QI8_S_ROW) == 0
    assert ops._gemm_ws_bytes(64, 3072, 3072, L.QI8_S_ROW, L.QI8_S_ROW) == 0
    assert ops._gemm_ws_bytes(64, 4096, 8192, L.QI8_S_ROW, L.QI8_S_ROW) > 0
    assert ops._gemm_ws_bytes(576, 3072, 15360, L.QI8_S_ROW, L.QI8_S_ROW) > 0
