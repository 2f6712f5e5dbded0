"""Pin the CPU oracle against the reference's own outputs (golden vectors).

Every fixture was produced by running the reference (its torch CPU path and
its Triton kernels under the Triton interpreter); see tests/golden/make_golden.py.
"""

import numpy as np
import pytest

import oracle as O


def test_fwht_rows_bitexact(golden):
    g = golden("fwht.npz")
    assert np.array_equal(O.fwht_rows(g["x1"]), g["y1"])
    assert np.array_equal(O.fwht_rows(g["x1"], normalize=False), g["y1n"])
    assert np.array_equal(O.fwht_rows(g["x2"]), g["y2"])
    assert np.array_equal(O.fwht_rows(g["x3"]), g["y3"])


def test_fwht_reference_gpu_kernel_matches_cpu_path(golden):
    # the reference's Triton per-stage kernels (interpreted) agree bit for bit
    # with its CPU core, so one oracle covers both reference paths
    g = golden("fwht.npz")
    assert np.array_equal(g["y2_triton"], g["y2"])
    signs = np.tile(g["s5c"], 4)
    assert np.array_equal(O.fwht_rows(g["x1"] * signs[None, :]), g["y1_triton_signs"])


def test_fwht_2d(golden):
    g = golden("fwht.npz")
    assert np.array_equal(O.fwht_2d(g["x5"]), g["y5_2d"])
    xs = g["x5"] * g["s5r"][:, None] * g["s5c"][None, :]
    assert np.array_equal(O.fwht_2d(xs), g["y5_2d_signs"])
    inv = O.fwht_2d(g["x5"]) * g["s5r"][:, None] * g["s5c"][None, :]
    assert np.array_equal(inv[:60, :100], g["y5_inv_2d_signs"])


def test_fwht_rejects_non_power_of_two():
    with pytest.raises(ValueError):
        O.fwht_rows(np.zeros((2, 12), np.float32))


def test_quantize_int8_axiswise_bitexact(golden):
    g = golden("act_token.npz")
    q, s = O.quantize_int8_axiswise(O.bf16_to_f32(g["xa_bf16"]))
    assert np.array_equal(q, g["qa"]) and np.array_equal(s, g["sa"])
    assert np.all(q[3] == 0) and s[3, 0] == np.float32(1e-30)
    q, s = O.quantize_int8_axiswise(g["xb"])
    assert np.array_equal(q, g["qb"]) and np.array_equal(s, g["sb"])


def test_rotate_quant_bitexact(golden):
    g = golden("rotate_quant.npz")
    x = O.bf16_to_f32(g["x_bf16"])
    xh = O.rotate_rows(x, g["s_v"], 4096)
    assert np.array_equal(xh, g["x_had"])
    q, s = O.rotate_quant_rows(x, g["s_v"], 4096)
    assert np.array_equal(q, g["q"]) and np.array_equal(s, g["s"])
    q2, s2 = O.rotate_quant_rows(O.bf16_to_f32(g["x2_bf16"]), g["s_v2"], 1024)
    assert np.array_equal(q2, g["q2"]) and np.array_equal(s2, g["s2"])


def test_quantize_int8_tensorwise_bitexact(golden):
    g = golden("tensorwise.npz")
    q, s = O.quantize_int8_tensorwise(O.bf16_to_f32(g["w_bf16"]))
    assert np.array_equal(q, g["q"]) and np.float32(s) == g["s"]


def test_triton_act_weight_quant(golden):
    g = golden("triton_quant.npz")
    y, s = O.act_quant(O.bf16_to_f32(g["x_bf16"]), 128)
    assert np.array_equal(y, g["y"]) and np.array_equal(s, g["s"])
    y2, s2 = O.act_quant(g["x2"], 128)
    assert np.array_equal(y2, g["y2"]) and np.array_equal(s2, g["s2"])
    qw, sw = O.weight_quant(g["w"], 128)
    assert np.array_equal(qw, g["qw"]) and np.array_equal(sw, g["sw"])
    assert np.array_equal(O.weight_dequant(g["qw"], g["sw"]), g["dw"])
    assert np.array_equal(O.act_dequant(g["y2"], g["s2"]), g["da2"])


def test_int_mm_bitexact(golden):
    g = golden("int_mm.npz")
    assert np.array_equal(O.int_mm(g["a"], g["b"]), g["c"])


@pytest.mark.parametrize("layout", ["tw", "aw"])
def test_linear_w8a8_bitexact(golden, layout):
    g = golden("linear.npz")
    x = O.bf16_to_f32(g["x_bf16"])
    bias = O.bf16_to_f32(g["bias_bf16"])
    wq, ws = g[f"{layout}_wq"], g[f"{layout}_ws"]
    x_q, x_s, acc, y = O.linear_w8a8(x, wq, ws, bias)
    assert np.array_equal(x_q, g[f"{layout}_xq"])
    assert np.array_equal(x_s, g[f"{layout}_xs"])
    assert np.array_equal(acc, g[f"{layout}_acc"])
    assert np.array_equal(O.f32_to_bf16(y), g[f"{layout}_y_bf16"])


def test_block_gemm_against_interpreted_kernel(golden):
    g = golden("gemm_block.npz")
    aq, bq = g["aq"], g["bq"]
    assert np.array_equal(O.act_quant(O.bf16_to_f32(g["x_bf16"]))[0], aq)
    c = O.int8_gemm_block(aq, g["a_s"], bq, g["b_s"], g["bias"]).astype(np.float16)
    ref = g["c_fp16"].view(np.float16)
    # the interpreted kernel's fp32 summation order inside tl.dot may differ;
    # the outputs agree to fp16 rounding
    rel = np.linalg.norm(c.astype(np.float32) - ref.astype(np.float32)) / np.linalg.norm(ref.astype(np.float32))
    assert rel < 1e-3
    c0 = O.int8_gemm_block(aq, g["a_s"], bq, g["b_s"], None).astype(np.float16)
    ref0 = g["c0_fp16"].view(np.float16)
    rel0 = np.linalg.norm(c0.astype(np.float32) - ref0.astype(np.float32)) / np.linalg.norm(ref0.astype(np.float32))
    assert rel0 < 1e-3


@pytest.mark.parametrize("tag,scheme,per_row", [("row", "tensor", True), ("glob", "tensor", False),
                                                ("block", "block", True)])
def test_quip_converter_pow2_bitexact(golden, tag, scheme, per_row):
    g = golden("quip_convert.npz")
    q, s, deq = O.quip_convert(g["w"], g["s_u"], g["s_v"], scheme, per_row)
    assert np.array_equal(q, g[f"{tag}_q"])
    assert np.array_equal(np.asarray(s).reshape(g[f"{tag}_s"].shape), g[f"{tag}_s"])
    assert np.array_equal(deq, g["row_deq"])


def test_quip_converter_store_transformed_bitexact(golden):
    g = golden("quip_convert.npz")
    q, s, deq = O.quip_convert(g["w"], g["s_u"], g["s_v"], store_transformed=True)
    assert np.array_equal(q, g["st_q"]) and np.array_equal(s, g["st_s"])
    assert np.array_equal(deq, g["st_deq"])
    assert int(g["st_hsize_out"]) == 128 and int(g["st_hsize_in"]) == 256


def test_quip_non_pow2_composition_bitexact(golden):
    g = golden("quip_convert.npz")
    w, su, sv = g["np_w"], g["np_s_u"], g["np_s_v"]
    wr = O.quip_rotate_weight(w, su, sv)
    assert np.array_equal(wr, g["np_wrot"])
    qr, sr = O.quip_rtn_rows(wr)
    assert np.array_equal(qr, g["np_qrot"]) and np.array_equal(sr, g["np_srot"])
    deq = O.quip_unrotate_weight(qr, sr, su, sv, 96, 192)
    assert np.array_equal(deq, g["np_deq"])
    q, s = O.quip_requant(deq, "tensor", True)
    assert np.array_equal(q, g["np_q_row"]) and np.array_equal(s, g["np_s_row"])
    qb, sb = O.quip_requant(deq, "block", True, block_size=64)
    assert np.array_equal(qb, g["np_q_block"]) and np.array_equal(sb, g["np_s_block"])


def test_quip_matmul_w8a8_close_to_reference_fp32(golden):
    # the reference's transformed-space matmul is fp32 (weights dequantized in
    # the kernel); the W8A8 restatement quantizes the rotated activations per
    # token, so it agrees to the north-star tolerance, not bit for bit
    g = golden("quip_matmul.npz")
    _, _, _, _, y = O.quip_linear_w8a8(g["x"], g["Q"], g["scale"], g["s_u"], g["s_v"], 128, None)
    ref = g["y"]
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert rel < 1e-2


def test_bf16_roundtrip():
    x = np.array([1.0, -2.5, 3.0e-3, 65504.0, 1.00390625, 1.01171875], np.float32)
    b = O.f32_to_bf16(x)
    assert np.array_equal(O.bf16_to_f32(b)[:4], np.array([1.0, -2.5, 0.0030059814453125, 65536.0], np.float32))
    # ties to even
    assert O.bf16_to_f32(b)[4] == np.float32(1.0) and O.bf16_to_f32(b)[5] == np.float32(1.015625)


def test_lpt_partition_balanced():
    costs = [10, 9, 8, 7, 6, 5, 4, 3, 2, 1]
    parts = O.lpt_partition(costs, 3)
    assert sorted(i for p in parts for i in p) == list(range(10))
    loads = [sum(costs[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= 2


def test_oracle_rotation_round_trip():
    r = np.random.default_rng(5)
    w = (r.standard_normal((100, 60)) * 0.02).astype(np.float32)
    su = (r.integers(0, 2, 128) * 2 - 1).astype(np.float32)
    sv = (r.integers(0, 2, 64) * 2 - 1).astype(np.float32)
    back = O.quip_inverse_rotate(O.quip_rotate_weight(w, su, sv), su, sv, 100, 60)
    assert np.max(np.abs(back - w)) < 1e-6


def test_fused_requant_gemm_and_int8_gelu_golden(golden):
    """int8_gemm_quant / int8_addmm_quant / int8_gelu (comfy/int8_kernels.py:
    684-1089, 1122-1312), executed by the reference under the Triton
    interpreter: int8 outputs and block scales bit-exact."""
    g = golden("gemm_quant.npz")
    q, s = O.int8_gemm_quant(g["aq"], g["a_s"], g["bq"], g["b_s"])
    assert np.array_equal(q, g["c_q"]) and np.array_equal(s, g["c_s"])
    q, s = O.int8_gemm_quant(g["aq"], g["a_s"], g["bq"], g["b_s"], g["bias"])
    assert np.array_equal(q, g["cb_q"]) and np.array_equal(s, g["cb_s"])
    q, s = O.int8_gelu(g["g_in_q"], g["g_in_s"])
    assert np.array_equal(q, g["g_q"]) and np.array_equal(s, g["g_s"])


def test_gptq_block_golden(golden):
    """gptq_quant_block_kernel (comfy/gptq_kernels.py:11-85) under the Triton
    interpreter: int8 codes, errors and the updated weight block bit-exact."""
    g = golden("gptq_block.npz")
    for tag in ("row", "scalar"):
        q, e, w = O.gptq_quant_block(g["w"], g["hinv"], g[f"{tag}_scale"])
        assert np.array_equal(q, g[f"{tag}_q"]) and np.array_equal(e, g[f"{tag}_err"])
        assert np.array_equal(w, g[f"{tag}_w_out"])


# ---------------------------------------------------------------- QuIP LDLQ
LDLQ_CASES = ("id", "wide", "cal", "blk", "st")


def ldlq_steps(g, tag):
    """The oracle's QuIP pass on a fixture case, with the permutations the
    reference drew (random) and sorted (act-order) taken from the fixture."""
    import torch
    w = g[f"{tag}_w"]
    M, N = w.shape
    H = g[f"{tag}_H"] if f"{tag}_H" in g else None
    s_u, s_v, perm = g[f"{tag}_s_u"], g[f"{tag}_s_v"], g[f"{tag}_perm"]
    D = g[f"{tag}_D"] if g[f"{tag}_D"].size else None
    if D is not None:
        wr, hr, D2 = O.diag_rescale(w, H)
    else:
        wr, hr, D2 = w, (np.eye(N, dtype=np.float32) if H is None else H), None
    Np = s_v.shape[0]
    wrot = O.quip_rotate_weight(wr, s_u, s_v)
    hpad = np.zeros((Np, Np), np.float32)
    hpad[:N, :N] = hr
    hrot = O.quip_rotate_weight(hpad, s_v, s_v)
    keys = O.damped_order_keys(hrot, perm)
    order = torch.argsort(torch.from_numpy(keys), descending=True).numpy()  # the reference's own sort
    wp, hp, damp = O.ldlq_prepare(wrot, hrot, perm, order)
    return dict(w=w, M=M, N=N, D=D, D2=D2, s_u=s_u, s_v=s_v, perm=perm, order=order, wp=wp, hp=hp, damp=damp,
                scale=O.quip_ldlq_scale(wp))


@pytest.mark.parametrize("tag", LDLQ_CASES)
def test_ldlq_oracle_pinned(golden, tag):
    g = golden("quip_ldlq.npz")
    st = ldlq_steps(g, tag)
    if st["D"] is not None:
        assert np.array_equal(st["D2"], st["D"])  # fp64 fourth root of the cascade column sums
    assert np.array_equal(st["order"], g[f"{tag}_order"])
    assert st["damp"] == g[f"{tag}_damp"]
    assert np.array_equal(st["wp"], g[f"{tag}_Wldlq"])
    assert np.array_equal(st["scale"], g[f"{tag}_scale"])
    if f"{tag}_Hinv" in g:
        hinv = O.ldlq_hinv(st["hp"])
        ref = g[f"{tag}_Hinv"]
        assert np.abs(hinv - ref).max() <= 1e-9 * np.abs(ref).max()
        assert (hinv == ref).mean() > 0.999
    else:
        hinv = O.ldlq_hinv(st["hp"])
    q = O.ldlq_pass(st["wp"], hinv, st["scale"], order="blas")
    assert np.array_equal(q, g[f"{tag}_Qldlq"])
    q_seq = O.ldlq_pass(st["wp"], hinv, st["scale"], order="seq")
    assert np.array_equal(q_seq, g[f"{tag}_Qldlq"])
    qo, deq = O.quip_ldlq_finish(g[f"{tag}_Qldlq"], st["scale"], st["perm"][st["order"]], st["s_u"], st["s_v"],
                                 st["M"], st["N"], st["D"])
    if tag == "st":
        assert np.array_equal(qo, g[f"{tag}_q"])
    else:
        assert np.array_equal(deq, g[f"{tag}_deq"])
        scheme = "block" if tag == "blk" else "tensor"
        q2, s2 = O.quip_requant(deq, scheme)
        assert np.array_equal(q2, g[f"{tag}_q"]) and np.array_equal(np.asarray(s2).reshape(-1),
                                                                    g[f"{tag}_s"].reshape(-1))


@pytest.mark.parametrize("shape", [(40, 600), (64, 600), (40, 8), (40, 7), (17, 600), (1, 9), (3000, 40),
                                   (5000, 5), (257, 1000), (96, 192)])
def test_col_sumsq_matches_torch_cpu_order(shape):
    """The cascade / row_sum grouping of torch's CPU sum, bit for bit."""
    import torch
    g = torch.Generator().manual_seed(shape[0] * 131 + shape[1])
    w = torch.randn(*shape, generator=g) * 0.02
    assert np.array_equal(O.col_sumsq(w.numpy()), (w ** 2).sum(dim=0).numpy())
