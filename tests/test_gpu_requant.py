"""GPU parity of the fused output requantization (int8_gemm_quant /
int8_addmm_quant, comfy/int8_kernels.py:684-1089) and the fused int8 GELU
(int8_gelu, :1122-1312) against the reference's own kernels (golden vectors
from the Triton interpreter) and the oracle at larger shapes.

Bar: int8 outputs and block scales bit-exact.  The GEMM's epilogue promotes
the K blocks in the reference's order, ``acc + (fp32(p) * a_s) * b_s``, so its
fp32 accumulator -- and hence the requantized int8 -- is reproduced exactly.
"""

import numpy as np
import pytest
import torch

import oracle as O
from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import ops
from convert_to_quant_quip_int8_b200.comfy import int8_kernels as IK
from convert_to_quant_quip_int8_b200.comfy import quant_ops as Q

pytestmark = pytest.mark.gpu


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def np_(t):
    return t.detach().cpu().numpy()


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    ops.device_status(reset=True)


def test_gemm_quant_golden(golden):
    g = golden("gemm_quant.npz")
    q, s = IK.int8_gemm_quant(cu(g["aq"]), cu(g["a_s"]), cu(g["bq"]), cu(g["b_s"]))
    assert np.array_equal(np_(q), g["c_q"]) and np.array_equal(np_(s), g["c_s"])
    q, s = IK.int8_addmm_quant(cu(g["aq"]), cu(g["a_s"]), cu(g["bq"]), cu(g["b_s"]), cu(g["bias"]))
    assert np.array_equal(np_(q), g["cb_q"]) and np.array_equal(np_(s), g["cb_s"])


def test_int8_gelu_golden(golden):
    g = golden("gemm_quant.npz")
    q, s = IK.int8_gelu(cu(g["g_in_q"]), cu(g["g_in_s"]))
    assert np.array_equal(np_(q), g["g_q"]) and np.array_equal(np_(s), g["g_s"])


def _block_case(M, N, K, seed, b_layout):
    r = np.random.default_rng(seed)
    x = r.standard_normal((M, K)).astype(np.float32)
    x[:, r.integers(0, K, 3)] *= 20.0
    aq, a_s = O.act_quant(x)
    w = (r.standard_normal((N, K)) * 0.02).astype(np.float32)
    if b_layout == "tile":
        bq, b_s = O.weight_quant(w)
    else:
        bq, b_s = O.quip_requant(w, "block")
        b_s = b_s.reshape(N, K // 128)
    bias = (r.standard_normal(N) * 0.1).astype(np.float32)
    return aq, a_s, bq, b_s, bias


@pytest.mark.parametrize("M,N,K", [(37, 256, 384), (128, 512, 1024), (300, 1024, 3072), (2048, 4096, 1024),
                                   (4096, 3072, 3072)])
@pytest.mark.parametrize("b_layout", ["tile", "row"])
def test_gemm_quant_vs_oracle(M, N, K, b_layout):
    """Single-CTA (M <= 128) and CTA-pair kernels, one wave and several waves
    of tiles (2048 x 4096: 128 pair tiles; 4096 x 3072: 192)."""
    aq, a_s, bq, b_s, bias = _block_case(M, N, K, M + N + K, b_layout)
    for b in (None, bias):
        q, s = ops.gemm_i8_quant(cu(aq), cu(bq), cu(a_s), cu(b_s), None if b is None else cu(b))
        q_ref, s_ref = O.int8_gemm_quant(aq, a_s, bq, b_s, b, b_layout=b_layout)
        assert np.array_equal(np_(s), s_ref)
        assert np.array_equal(np_(q), q_ref)


@pytest.mark.parametrize("rows,n", [(1, 128), (300, 1024), (4096, 3072), (4096, 12288)])
def test_int8_gelu_vs_oracle(rows, n):
    r = np.random.default_rng(rows + n)
    x = (r.standard_normal((rows, n)) * 3.0).astype(np.float32)
    q, s = O.act_quant(x)
    qo, so = ops.int8_gelu(cu(q), cu(s))
    q_ref, s_ref = O.int8_gelu(q, s)
    assert np.array_equal(np_(so), s_ref)
    assert np.array_equal(np_(qo), q_ref)


def test_blockwise_handlers_out_quant():
    """The BlockWiseINT8Layout linear / addmm handlers with out_quant=True
    return int8 QuantizedTensors from the fused kernel (comfy/quant_ops.py:
    373-417), and aten.gelu on such a tensor runs the fused int8 GELU."""
    aq, a_s, bq, b_s, bias = _block_case(200, 512, 768, 5, "tile")
    xq = Q.QuantizedTensor(cu(aq), "BlockWiseINT8Layout", {"scale": cu(a_s), "block_size": 128, "is_weight": False,
                                                            "orig_dtype": torch.bfloat16})
    wq = Q.QuantizedTensor(cu(bq), "BlockWiseINT8Layout", {"scale": cu(b_s), "block_size": 128, "is_weight": True,
                                                            "orig_dtype": torch.bfloat16})
    handler = Q._LAYOUT_REGISTRY[torch.ops.aten.linear.default]["BlockWiseINT8Layout"]
    y = handler(torch.ops.aten.linear.default, (xq, wq, cu(bias)), {"out_quant": True})
    q_ref, s_ref = O.int8_gemm_quant(aq, a_s, bq, b_s, bias)
    assert isinstance(y, Q.QuantizedTensor) and y._layout_params["block_size"] == 128
    assert np.array_equal(np_(y._qdata), q_ref) and np.array_equal(np_(y._layout_params["scale"]), s_ref)
    g = Q._LAYOUT_REGISTRY[torch.ops.aten.gelu.default]["BlockWiseINT8Layout"](torch.ops.aten.gelu.default, (y,), {})
    gq_ref, gs_ref = O.int8_gelu(q_ref, s_ref)
    assert np.array_equal(np_(g._qdata), gq_ref) and np.array_equal(np_(g._layout_params["scale"]), gs_ref)


def test_gemm_quant_rejects_unsupported():
    aq, a_s, bq, b_s, _ = _block_case(64, 256, 256, 1, "tile")
    with pytest.raises(AssertionError):  # N not a multiple of the 128-column output block
        ops.gemm_i8_quant(cu(aq), cu(bq[:144]), cu(a_s), cu(b_s[:2]))
    lib = L.load()
    q = torch.empty(64, 256, dtype=torch.int8, device="cuda")
    s = torch.empty(64, 2, device="cuda")
    xs = torch.ones(64, 1, device="cuda")
    # per-token activation scales are not the block format this kernel requantizes from
    with pytest.raises(AssertionError):
        L.check(lib.qi8_gemm_i8_quant(L.ptr(cu(aq)), L.ptr(cu(bq)), 64, 256, 256, L.ptr(xs), L.QI8_S_ROW,
                                      L.ptr(cu(b_s)), L.QI8_S_TILE128, None, 0, L.ptr(q), 256, L.ptr(s), 128,
                                      L.stream_ptr()), "qi8_gemm_i8_quant")
    with pytest.raises(AssertionError):  # output block other than 128
        L.check(lib.qi8_gemm_i8_quant(L.ptr(cu(aq)), L.ptr(cu(bq)), 64, 256, 256, L.ptr(cu(a_s)),
                                      L.QI8_S_ROW_KBLOCK, L.ptr(cu(b_s)), L.QI8_S_TILE128, None, 0, L.ptr(q), 256,
                                      L.ptr(s), 64, L.stream_ptr()), "qi8_gemm_i8_quant")
    with pytest.raises(AssertionError):
        IK.int8_gelu(cu(aq)[:, :100].contiguous(), cu(a_s)[:, :1].contiguous())
