"""GPU parity at the benchmarked sizes.

Every case here runs a workload's real shape, so the persistent tcgen05 GEMM
walks several output tiles per CTA pair (tile-index advance, TMEM buffer
hand-off across tiles, barrier phases carried over) and K1 runs its
persistent row-group loop over thousands of rows.  Each result is compared
with the CPU oracle on the same seeded inputs:

* the DiT MLP pair (4096 tokens): W1 [12288, 3072] and W2 [3072, 12288] with
  block-128 ``[N, K/128]`` weight scales and per-token activation scales --
  fp32 output within rel 1e-5 of the oracle's block-promoted GEMM (the int32
  partials are exact; only the fp32 summation order differs), bf16 within
  1e-2, and the int32 accumulators of both shapes bit-exact;
* the single QuIP linear (512 x 4096 -> 4096, transformed storage):
  K1 -> K2 -> K3, every stage bit-exact;
* one Flux single-block linear (4608 x 3072 -> 21504, per-row scale, bias)
  and one T5-XXL wi linear (4096 x 10240 -> 4096, axis-wise scale):
  per-token int8, int32 accumulator and bf16 output bit-exact.
"""

import numpy as np
import pytest
import torch

import oracle as O
from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import ops
from convert_to_quant_quip_int8_b200.workloads import DitMlpPair, SingleQuipLinear, normal, student_t_outliers, gen

pytestmark = pytest.mark.gpu

REL_BF16 = 1e-2
REL_F32_BLOCK = 1e-5


def dev():
    return torch.device("cuda", 0)


def np_(t):
    return t.detach().cpu().numpy()


def bf16_bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def rel_fro(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    ops.device_status(reset=True)


@pytest.fixture(scope="module")
def dit():
    """The DiT MLP pair exactly as the benchmark builds it: W1 QuIP-converted
    with block requant on the GPU, W2 block-requantized, x quantized per token."""
    wl = DitMlpPair()
    su, sv = wl.w1_signs()
    q1, s1, _ = ops.quip_convert(wl.w1().to(dev()), su, sv, requant=L.QI8_REQ_BLOCK, want_dequant=False)
    q2, s2 = ops.requant_weight(wl.w2().to(dev()), L.QI8_REQ_BLOCK)
    x = wl.activations()
    xq, xs = ops.quant_rows(x.to(dev()), L.QI8_Q_TOKEN)
    torch.cuda.synchronize()
    return dict(wl=wl, x=x, xq=xq, xs=xs, q1=q1, s1=s1.reshape(q1.shape[0], -1).contiguous(),
                q2=q2, s2=s2.reshape(q2.shape[0], -1).contiguous())


def test_dit_activation_quant_fullsize(dit):
    xq_ref, xs_ref = O.quantize_int8_axiswise(dit["x"].float().numpy())
    assert np.array_equal(np_(dit["xq"]), xq_ref)
    assert np.array_equal(np_(dit["xs"]).reshape(-1), xs_ref.reshape(-1))


def test_dit_w1_conversion_fullsize(dit):
    """W1's QuIP conversion (12288 x 3072, padded 16384 x 4096) against the
    oracle converter: quantized weight and block scales bit-exact."""
    wl = dit["wl"]
    su, sv = (t.numpy() for t in wl.w1_signs())
    q_ref, s_ref, _ = O.quip_convert(wl.w1().float().numpy(), su, sv, "block")
    assert np.array_equal(np_(dit["q1"]), q_ref)
    assert np.array_equal(np_(dit["s1"]).reshape(-1), np.asarray(s_ref).reshape(-1))


@pytest.mark.parametrize("which", ["w1", "w2"])
def test_dit_block_gemm_fullsize(dit, which):
    """4096 x 3072 -> 12288 (W1) and 4096 x 12288 -> 3072 (W2): 16 x 48 and
    16 x 12 output tiles of 256 x 256, i.e. several tiles per CTA pair."""
    if which == "w1":
        a, a_s = dit["xq"], dit["xs"]
        b, b_s = dit["q1"], dit["s1"]
    else:
        # the W2 input is GELU(W1 output) quantized per token by K1 (GELU fused)
        h = ops.gemm_i8(dit["xq"], dit["q1"], dit["xs"], L.QI8_S_ROW, dit["s1"], L.QI8_S_ROW_KBLOCK, None,
                        torch.bfloat16)
        a, a_s = ops.quant_rows(h, L.QI8_Q_TOKEN | L.QI8_Q_GELU)
        b, b_s = dit["q2"], dit["s2"]
    an, asn, bn, bsn = np_(a), np_(a_s), np_(b), np_(b_s)
    ref = O.int8_gemm_block(an, asn, bn, bsn, None, b_layout="row")
    y32 = ops.gemm_i8(a, b, a_s, L.QI8_S_ROW, b_s, L.QI8_S_ROW_KBLOCK, None, torch.float32)
    assert rel_fro(np_(y32), ref) < REL_F32_BLOCK
    y16 = ops.gemm_i8(a, b, a_s, L.QI8_S_ROW, b_s, L.QI8_S_ROW_KBLOCK, None, torch.bfloat16)
    assert rel_fro(np_(y16.float()), ref) < REL_BF16
    del ref, y32, y16
    acc = ops.gemm_i8(a, b, out_dtype=torch.int32)
    assert np.array_equal(np_(acc), O.int_mm(an, bn))


def test_quip_linear_config1_fullsize():
    """Config 1 at full size: x [512, 4096], W' [4096, 4096] transformed
    storage; K1 (signs + FWHT + per-token int8), K2 (fp32 out), K3 (FWHT +
    signs + bias -> bf16)."""
    wl = SingleQuipLinear()
    su, sv = wl.signs()
    q, s, _ = ops.quip_convert(wl.weight().to(dev()), su, sv, store_transformed=True, want_dequant=False)
    q_ref, s_ref, _ = O.quip_convert(wl.weight().float().numpy(), su.numpy(), sv.numpy(), store_transformed=True)
    assert np.array_equal(np_(q), q_ref)
    assert np.array_equal(np_(s).reshape(-1), np.asarray(s_ref).reshape(-1))
    x = wl.activations()
    bias = wl.bias()
    D = wl.dim
    xq, xs = ops.rotate_quant_rows(x.to(dev()), sv.to(dev()), D)
    y_had = ops.gemm_i8(xq, q, xs, L.QI8_S_ROW, s, L.QI8_S_ROW, None, torch.float32)
    y = ops.unrotate_rows(y_had, su.to(dev()), D, bias.to(dev()), torch.bfloat16)
    xq_r, xs_r, acc_r, yh_r, y_r = O.quip_linear_w8a8(x.float().numpy(), q_ref, np.asarray(s_ref).reshape(-1),
                                                      su.numpy(), sv.numpy(), D, bias.float().numpy())
    assert np.array_equal(np_(xq), xq_r)
    assert np.array_equal(np_(xs).reshape(-1), xs_r.reshape(-1))
    assert np.array_equal(np_(y_had), yh_r)
    assert np.array_equal(bf16_bits(y), O.f32_to_bf16(y_r))
    assert np.array_equal(np_(ops.gemm_i8(xq, q, out_dtype=torch.int32)), acc_r)


def _linear_case(T, K, N, x_seed, w_seed, bias, heavy_tail=False):
    x = normal((T, K), 1.0, x_seed)
    if heavy_tail:
        x = student_t_outliers(x, 0.01, 3, x_seed + 1)
    x = x.to(torch.bfloat16)
    w = (torch.randn(N, K, generator=gen(w_seed)) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=gen(w_seed + 1)) * 0.01).to(torch.bfloat16) if bias else None
    return x, w, b


@pytest.mark.parametrize("name,T,K,N,bias,heavy", [
    ("flux_single_linear1", 4608, 3072, 21504, True, False),
    ("t5_wi", 4096, 4096, 10240, False, True),
    ("t5_wo", 4096, 10240, 4096, False, True),
])
def test_w8a8_linear_fullsize_bitexact(name, T, K, N, bias, heavy):
    """Per-token W8A8 linear with a per-output-row weight scale: the Flux
    stack's per-row [N, 1] QuIP scale and T5's axis-wise [N] scale are the
    same epilogue (comfy/quant_ops.py:472-474)."""
    x, w, b = _linear_case(T, K, N, 300 + K, 400 + N, bias, heavy)
    wq, ws = ops.quant_weight(w.to(dev()), L.QI8_S_ROW)
    wq_r, ws_r = O.quantize_int8_axiswise(w.float().numpy())
    assert np.array_equal(np_(wq), wq_r)
    assert np.array_equal(np_(ws).reshape(-1), ws_r.reshape(-1))
    xd = x.to(dev())
    xq, xs = ops.quant_rows(xd, L.QI8_Q_TOKEN)
    bd = None if b is None else b.to(dev())
    y = ops.gemm_i8(xq, wq, xs, L.QI8_S_ROW, ws.reshape(-1), L.QI8_S_ROW, bd, torch.bfloat16)
    xq_r, xs_r, acc_r, y_r = O.linear_w8a8(x.float().numpy(), wq_r, ws_r.reshape(-1),
                                           None if b is None else b.float().numpy())
    assert np.array_equal(np_(xq), xq_r)
    assert np.array_equal(np_(xs).reshape(-1), xs_r.reshape(-1))
    assert np.array_equal(bf16_bits(y), O.f32_to_bf16(y_r))
    assert np.array_equal(np_(ops.gemm_i8(xq, wq, out_dtype=torch.int32)), acc_r)
