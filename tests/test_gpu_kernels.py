"""GPU parity of the libqi8 kernels against the CPU oracle and the golden
vectors produced by the reference itself.

Bars (north star): int8 tensors, int32 accumulators and quantized weights
bit-exact; FWHT outputs bit-exact (stricter than the 1e-3 relative bar);
dequantized bf16 outputs within 1e-2 relative Frobenius error.
"""

import numpy as np
import pytest
import torch

import oracle as O
from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import ops

pytestmark = pytest.mark.gpu

REL_BF16 = 1e-2


def dev():
    return torch.device("cuda", 0)


def cu(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(dev())


def bf16_cu(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev())


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


def rng(seed):
    return np.random.default_rng(seed)


# ----------------------------------------------------------------- FWHT
@pytest.mark.parametrize("L2", list(range(1, 16)))
def test_fwht_rows_bitexact_all_sizes(L2):
    n = 1 << L2
    rows = 3 if n >= 8192 else 7
    x = rng(L2).standard_normal((rows, n)).astype(np.float32)
    y = ops.fwht_rows(cu(x))
    assert np.array_equal(np_(y), O.fwht_rows(x))
    yn = ops.fwht_rows(cu(x), normalize=False)
    assert np.array_equal(np_(yn), O.fwht_rows(x, normalize=False))


def test_fwht_golden(golden):
    g = golden("fwht.npz")
    assert np.array_equal(np_(ops.fwht_rows(cu(g["x1"]))), g["y1"])
    assert np.array_equal(np_(ops.fwht_rows(cu(g["x1"]), normalize=False)), g["y1n"])
    assert np.array_equal(np_(ops.fwht_rows(cu(g["x2"]))), g["y2"])
    assert np.array_equal(np_(ops.fwht_rows(cu(g["x3"]))), g["y3"])


def test_fwht_signs_and_padding_bf16():
    r = rng(5)
    x = r.standard_normal((9, 3072)).astype(np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16)
    s1 = (r.integers(0, 2, 4096) * 2 - 1).astype(np.float32)
    s2 = (r.integers(0, 2, 4096) * 2 - 1).astype(np.float32)
    y = ops.fwht_rows(xb.to(dev()), n_pad=4096, pre_sign=cu(s1), post_sign=cu(s2))
    ref = O.rotate_rows(xb.float().numpy(), s1, 4096) * s2[None, :]
    assert np.array_equal(np_(y), ref)


# -------------------------------------------------------- per-token quant
def test_quant_rows_token_golden(golden):
    g = golden("act_token.npz")
    q, s = ops.quant_rows(bf16_cu(g["xa_bf16"]))
    assert np.array_equal(np_(q), g["qa"]) and np.array_equal(np_(s), g["sa"])
    q, s = ops.quant_rows(cu(g["xb"]))  # n = 1000
    assert np.array_equal(np_(q), g["qb"]) and np.array_equal(np_(s), g["sb"])


@pytest.mark.parametrize("n", [8, 128, 3072, 4096, 10240, 12288, 15360, 32768])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quant_rows_token_random(n, dtype):
    r = rng(n)
    x = r.standard_normal((13, n)).astype(np.float32) * 3
    x[:, r.integers(0, n, 3)] *= 40
    xt = torch.from_numpy(x).to(dtype)
    q, s = ops.quant_rows(xt.to(dev()))
    qr, sr = O.quantize_int8_axiswise(xt.float().numpy())
    assert np.array_equal(np_(q), qr) and np.array_equal(np_(s), sr)


@pytest.mark.parametrize("n,rows", [(3072, 3000), (12288, 2049), (24576, 300)])
def test_quant_rows_token_many_rows(n, rows):
    # more row groups than resident blocks: the persistent loop, plus a zero
    # row and a one-hot row
    r = rng(n + rows)
    x = (r.standard_normal((rows, n)) * 2).astype(np.float32)
    x[5] = 0.0
    x[7] = 0.0
    x[7, n - 1] = -3.0
    xt = torch.from_numpy(x).to(torch.bfloat16)
    q, s = ops.quant_rows(xt.to(dev()))
    qr, sr = O.quantize_int8_axiswise(xt.float().numpy())
    assert np.array_equal(np_(q), qr) and np.array_equal(np_(s), sr)


@pytest.mark.parametrize("n", [3072, 12288, 1000, 24576])
def test_quant_rows_gelu_fused(n):
    # GELU between the DiT MLP projections: torch gelu on the bf16 tensor, then per-token quant
    r = rng(n + 1)
    h = torch.from_numpy((r.standard_normal((9, n)) * 2).astype(np.float32)).to(torch.bfloat16)
    q, s = ops.quant_rows(h.to(dev()), L.QI8_Q_TOKEN | L.QI8_Q_GELU)
    g = torch.nn.functional.gelu(h.float()).to(torch.bfloat16).float().numpy()
    qr, sr = O.quantize_int8_axiswise(g)
    # erff (CUDA) vs erf (CPU) may differ in the last ulp before the bf16 rounding
    assert np.mean(np_(q) != qr) < 1e-3 and np.max(np.abs(np_(q).astype(int) - qr)) <= 1
    assert np.allclose(np_(s), sr, rtol=1e-2)


@pytest.mark.parametrize("n", [3072, 12288])
def test_quant_rows_gelu_equals_torch_gelu_then_quant(n):
    # the fused GELU reproduces torch's bf16 F.gelu on the GPU bit for bit
    r = rng(n + 7)
    h = torch.from_numpy((r.standard_normal((257, n)) * 3).astype(np.float32)).to(torch.bfloat16).to(dev())
    q, s = ops.quant_rows(h, L.QI8_Q_TOKEN | L.QI8_Q_GELU)
    q2, s2 = ops.quant_rows(torch.nn.functional.gelu(h), L.QI8_Q_TOKEN)
    assert torch.equal(q, q2) and torch.equal(s, s2)


def test_quant_rows_gelu_every_bf16_value():
    # one finite bf16 value per row (the rest zeros): the row scale exposes
    # GELU of that value, so every bf16 input -- table range and outside it --
    # is checked against torch's bf16 F.gelu
    bits = torch.arange(65536, dtype=torch.int32)
    bits = bits[((bits >> 7) & 0xFF) != 0xFF].to(torch.int16)
    v = bits.view(torch.bfloat16)
    h = torch.zeros(v.numel(), 16, dtype=torch.bfloat16)
    h[:, 0] = v
    h[:, 9] = v
    h = h.to(dev())
    q, s = ops.quant_rows(h, L.QI8_Q_TOKEN | L.QI8_Q_GELU)
    q2, s2 = ops.quant_rows(torch.nn.functional.gelu(h), L.QI8_Q_TOKEN)
    assert torch.equal(q, q2) and torch.equal(s, s2)


def test_quant_rows_block_golden(golden):
    g = golden("triton_quant.npz")
    q, s = ops.quant_rows(bf16_cu(g["x_bf16"]), mode=L.QI8_Q_BLOCK)
    assert np.array_equal(np_(q), g["y"]) and np.array_equal(np_(s), g["s"])
    q, s = ops.quant_rows(cu(g["x2"]), mode=L.QI8_Q_BLOCK)
    assert np.array_equal(np_(q), g["y2"]) and np.array_equal(np_(s), g["s2"])


def test_quant_rows_strided_input():
    r = rng(9)
    x = torch.from_numpy(r.standard_normal((6, 4096)).astype(np.float32)).to(dev())
    view = x[:, :3072]  # row stride 4096 != width
    q, s = ops.quant_rows(view)
    qr, sr = O.quantize_int8_axiswise(np_(view))
    assert np.array_equal(np_(q), qr) and np.array_equal(np_(s), sr)


# ---------------------------------------------------------- K1 rotate+quant
def test_rotate_quant_golden(golden):
    g = golden("rotate_quant.npz")
    q, s = ops.rotate_quant_rows(bf16_cu(g["x_bf16"]), cu(g["s_v"]), 4096)
    assert np.array_equal(np_(q), g["q"]) and np.array_equal(np_(s), g["s"])
    q2, s2 = ops.rotate_quant_rows(bf16_cu(g["x2_bf16"]), cu(g["s_v2"]), 1024)
    assert np.array_equal(np_(q2), g["q2"]) and np.array_equal(np_(s2), g["s2"])


@pytest.mark.parametrize("n,n_pad", [(3072, 4096), (4096, 4096), (12288, 16384), (15360, 16384),
                                     (21504, 32768), (100, 128), (9216, 16384), (10240, 16384)])
def test_rotate_quant_random(n, n_pad):
    r = rng(n + n_pad)
    rows = 5
    x = r.standard_normal((rows, n)).astype(np.float32)
    x[:, r.integers(0, n, 4)] *= 20
    xb = torch.from_numpy(x).to(torch.bfloat16)
    sv = (r.integers(0, 2, n_pad) * 2 - 1).astype(np.float32)
    q, s = ops.rotate_quant_rows(xb.to(dev()), cu(sv), n_pad)
    qr, sr = O.rotate_quant_rows(xb.float().numpy(), sv, n_pad)
    assert np.array_equal(np_(q), qr) and np.array_equal(np_(s), sr)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rotate_quant_two_phase_n4096(dtype):
    """The two-phase n = 4096 kernel (16-bit rows whose width is a multiple
    of 64) against the oracle on 2500 rows (several rows per persistent
    CTA), with outlier channels, an all-zero row and, in bf16, rows whose
    amax leaves the folded-normalization range; then against the phased
    kernel (a 3000-wide row takes it) on the same data with and without
    signs and normalization, and with signs other than +-1."""
    r = rng(4096)
    rows, n = 2500, 3072
    x = r.standard_normal((rows, n)).astype(np.float32)
    x[:, r.integers(0, n, 8)] *= 30
    x[3] = 0
    if dtype == torch.bfloat16:
        x[5] *= 1e31
        x[6] *= 1e-34
    else:
        x[5] *= 100
        x[6] *= 1e-3
    xt = torch.from_numpy(x).to(dtype)
    sv = (r.integers(0, 2, 4096) * 2 - 1).astype(np.float32)
    q, s = ops.rotate_quant_rows(xt.to(dev()), cu(sv), 4096)
    qr, sr = O.rotate_quant_rows(xt.float().numpy(), sv, 4096)
    assert np.array_equal(np_(q), qr) and np.array_equal(np_(s).reshape(-1), sr.reshape(-1))
    xz = xt.clone()
    xz[:, 3000:] = 0
    # signs other than +-1 take the multiply path instead of the sign-bit flip
    sw = (sv * r.uniform(0.5, 2.0, 4096)).astype(np.float32)
    qw, sw_ = ops.rotate_quant_rows(xt.to(dev()), cu(sw), 4096)
    qwr, swr = O.rotate_quant_rows(xt.float().numpy(), sw, 4096)
    assert np.array_equal(np_(qw), qwr) and np.array_equal(np_(sw_).reshape(-1), swr.reshape(-1))
    for sign, norm in ((cu(sv), True), (None, True), (cu(sv), False), (None, False), (cu(sw), True)):
        q1, s1 = ops.rotate_quant_rows(xz.to(dev()), sign, 4096, normalize=norm)
        q2, s2 = ops.rotate_quant_rows(xz[:, :3000].contiguous().to(dev()), sign, 4096, normalize=norm)
        assert torch.equal(q1, q2) and torch.equal(s1, s2), (sign is None, norm)


def test_rotate_quant_block_mode():
    r = rng(77)
    x = torch.from_numpy(r.standard_normal((4, 3072)).astype(np.float32)).to(torch.bfloat16)
    sv = (r.integers(0, 2, 4096) * 2 - 1).astype(np.float32)
    q, s = ops.rotate_quant_rows(x.to(dev()), cu(sv), 4096, mode=L.QI8_Q_BLOCK)
    qr, sr = O.act_quant(O.rotate_rows(x.float().numpy(), sv, 4096), 128)
    assert np.array_equal(np_(q), qr) and np.array_equal(np_(s), sr)


def test_rotate_rejects_non_pow2():
    with pytest.raises(ValueError):
        ops.rotate_quant_rows(torch.zeros(2, 12, device=dev()), None, 12)


# ------------------------------------------------------------ K3 unrotate
@pytest.mark.parametrize("n_out,n_pad", [(4096, 4096), (3072, 4096), (9216, 16384)])
def test_unrotate_rows(n_out, n_pad):
    r = rng(n_out)
    y = r.standard_normal((6, n_pad)).astype(np.float32)
    su = (r.integers(0, 2, n_pad) * 2 - 1).astype(np.float32)
    bias = torch.from_numpy(r.standard_normal(n_out).astype(np.float32) * 0.01).to(torch.bfloat16)
    out = ops.unrotate_rows(cu(y), cu(su), n_out, bias.to(dev()), torch.bfloat16)
    ref = O.unrotate_rows(y, su, n_out, bias.float().numpy())
    assert np.array_equal(bf16_bits(out), O.f32_to_bf16(ref))


# ------------------------------------------------------------------ GEMM
def test_gemm_int32_golden(golden):
    g = golden("int_mm.npz")
    c = ops.gemm_i8(cu(g["a"]), cu(g["b"]), out_dtype=torch.int32)
    assert np.array_equal(np_(c), g["c"])


@pytest.mark.parametrize("M,N,K", [(1, 16, 16), (37, 80, 256), (128, 256, 128), (129, 272, 336),
                                   (300, 512, 4096), (1024, 1024, 1024), (64, 3072, 12288), (515, 784, 208)])
def test_gemm_int32_bitexact(M, N, K):
    r = rng(M * 7 + N * 3 + K)
    a = r.integers(-128, 128, (M, K), dtype=np.int8)
    b = r.integers(-128, 128, (N, K), dtype=np.int8)
    c = ops.gemm_i8(cu(a), cu(b), out_dtype=torch.int32)
    assert np.array_equal(np_(c), O.int_mm(a, b))


def test_gemm_int32_extremes():
    # all -128: the largest magnitude accumulator (128*128*K)
    K = 16384
    a = np.full((128, K), -128, np.int8)
    b = np.full((256, K), -128, np.int8)
    c = ops.gemm_i8(cu(a), cu(b), out_dtype=torch.int32)
    assert np.all(np_(c) == 128 * 128 * K)


@pytest.mark.parametrize("layout", ["tw", "aw"])
def test_linear_epilogue_golden_bitexact(golden, layout):
    g = golden("linear.npz")
    xq, xs = cu(g[f"{layout}_xq"]), cu(g[f"{layout}_xs"])
    wq, ws = cu(g[f"{layout}_wq"]), cu(g[f"{layout}_ws"])
    bias = bf16_cu(g["bias_bf16"])
    kind = L.QI8_S_SCALAR if layout == "tw" else L.QI8_S_ROW
    y = ops.gemm_i8(xq, wq, xs, L.QI8_S_ROW, ws, kind, bias, torch.bfloat16)
    assert np.array_equal(bf16_bits(y), g[f"{layout}_y_bf16"])


def test_gemm_block_tile_golden(golden):
    g = golden("gemm_block.npz")
    y = ops.gemm_i8(cu(g["aq"]), cu(g["bq"]), cu(g["a_s"]), L.QI8_S_ROW_KBLOCK, cu(g["b_s"]), L.QI8_S_TILE128,
                    cu(g["bias"]), torch.float16)
    ref = g["c_fp16"].view(np.float16).astype(np.float32)
    assert rel_fro(np_(y).astype(np.float32), ref) < 1e-3
    y32 = ops.gemm_i8(cu(g["aq"]), cu(g["bq"]), cu(g["a_s"]), L.QI8_S_ROW_KBLOCK, cu(g["b_s"]), L.QI8_S_TILE128,
                      cu(g["bias"]), torch.float32)
    ref32 = O.int8_gemm_block(g["aq"], g["a_s"], g["bq"], g["b_s"], g["bias"])
    assert rel_fro(np_(y32), ref32) < 1e-5


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (300, 1024, 3072), (128, 3072, 12288)])
def test_gemm_block_rowk_per_token(M, N, K):
    # QuIP block requant weights ([N, K/128, 1] scales) x per-token activations
    r = rng(M + N + K)
    a = r.integers(-128, 128, (M, K), dtype=np.int8)
    b = r.integers(-127, 128, (N, K), dtype=np.int8)
    sa = (r.random((M, 1)) * 0.05 + 0.01).astype(np.float32)
    sb = (r.random((N, K // 128, 1)) * 1e-3 + 1e-4).astype(np.float32)
    bias = (r.standard_normal(N) * 0.01).astype(np.float32)
    y = ops.gemm_i8(cu(a), cu(b), cu(sa), L.QI8_S_ROW, cu(sb), L.QI8_S_ROW_KBLOCK, cu(bias), torch.float32)
    ref = O.int8_gemm_block(a, sa, b, sb.reshape(N, -1), bias, b_layout="row")
    assert rel_fro(np_(y), ref) < 1e-5
    yb = ops.gemm_i8(cu(a), cu(b), cu(sa), L.QI8_S_ROW, cu(sb), L.QI8_S_ROW_KBLOCK, cu(bias), torch.bfloat16)
    assert rel_fro(np_(yb.float()), ref) < REL_BF16


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (300, 1040, 2048), (129, 272, 336), (1000, 1040, 1024),
                                   (2048, 3072, 3072)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gemm_few_tiles_epilogue_bitexact(M, N, K, dtype):
    """Plain per-row GEMMs whose 256-column pair tiles would fill at most a
    quarter of the CTA pairs run 128-column tiles (ragged last tile at
    N = 1040); 512 x 4096 (32 tiles) and 2048 x 3072 keep 256-column tiles.
    Output with bias is bit-exact against the oracle's W8A8 epilogue."""
    r = rng(M + 3 * N + K)
    a = r.integers(-128, 128, (M, K), dtype=np.int8)
    b = r.integers(-127, 128, (N, K), dtype=np.int8)
    sa = (r.random((M, 1)) * 0.01 + 1e-3).astype(np.float32)
    sb = (r.random(N) * 1e-3 + 1e-4).astype(np.float32)
    bias = torch.from_numpy((r.standard_normal(N) * 0.1).astype(np.float32)).to(torch.bfloat16)
    y = ops.gemm_i8(cu(a), cu(b), cu(sa), L.QI8_S_ROW, cu(sb), L.QI8_S_ROW, bias.to(dev()), dtype)
    ref = O.linear_w8a8_epilogue(O.int_mm(a, b), sa, sb, bias.float().numpy())
    if dtype == torch.bfloat16:
        assert np.array_equal(bf16_bits(y), O.f32_to_bf16(ref))
    else:
        assert np.array_equal(np_(y), ref)


@pytest.mark.parametrize("M,N,K,dtype,bias,act", [
    (64, 3072, 1024, torch.bfloat16, True, L.QI8_ACT_NONE),     # one 64-token tile
    (64, 3072, 512, torch.bfloat16, True, L.QI8_ACT_GELU),
    (40, 1024, 256, torch.bfloat16, False, L.QI8_ACT_NONE),
    (1, 512, 2048, torch.bfloat16, True, L.QI8_ACT_NONE),
    (33, 1040, 256, torch.float16, False, L.QI8_ACT_NONE),      # ragged features: the last lane tile holds 16
    (576, 3072, 1024, torch.bfloat16, True, L.QI8_ACT_NONE),    # more than 128 tokens stay on the lanes
])
def test_gemm_weights_on_lanes_bitexact(M, N, K, dtype, bias, act):
    """Unsplit plain GEMMs of at most 64 tokens run with the weights on the
    TMEM lanes and the tokens as a 64-wide tile, stored through a per-warp
    transpose.  Every output equals the
    tokens-on-lanes kernel's (the same tokens zero-padded to a multiple of
    256 rows, which keeps them on the lanes) bit for bit, and without GELU
    the oracle's epilogue in bf16/f16."""
    r = rng(M + 5 * N + K)
    a = r.integers(-128, 128, (M, K), dtype=np.int8)
    b = r.integers(-127, 128, (N, K), dtype=np.int8)
    sa = (r.random((M, 1)) * 0.01 + 1e-3).astype(np.float32)
    sb = (r.random(N) * 1e-3 + 1e-4).astype(np.float32)
    bt = torch.from_numpy((r.standard_normal(N) * 0.1).astype(np.float32)).to(torch.bfloat16) if bias else None
    y = ops.gemm_i8(cu(a), cu(b), cu(sa), L.QI8_S_ROW, cu(sb), L.QI8_S_ROW,
                    None if bt is None else bt.to(dev()), dtype, act=act)
    Mp = (M + 255) // 256 * 256
    ap = np.zeros((Mp, K), np.int8)
    ap[:M] = a
    sap = np.full((Mp, 1), 1e-3, np.float32)
    sap[:M] = sa
    yl = ops.gemm_i8(cu(ap), cu(b), cu(sap), L.QI8_S_ROW, cu(sb), L.QI8_S_ROW,
                     None if bt is None else bt.to(dev()), dtype, act=act)
    assert torch.equal(y, yl[:M])
    if act == L.QI8_ACT_GELU:
        return
    ref = O.linear_w8a8_epilogue(O.int_mm(a, b), sa, sb, None if bt is None else bt.float().numpy())
    if dtype == torch.bfloat16:
        assert np.array_equal(bf16_bits(y), O.f32_to_bf16(ref))
    else:
        assert np.array_equal(np_(y).view(np.uint16), ref.astype(np.float16).view(np.uint16))


def test_gemm_gelu_epilogue():
    r = rng(3)
    M, N, K = 200, 512, 512
    a = r.integers(-128, 128, (M, K), dtype=np.int8)
    b = r.integers(-127, 128, (N, K), dtype=np.int8)
    sa = (r.random((M, 1)) * 0.01).astype(np.float32)
    sb = (r.random((N, 1)) * 1e-3).astype(np.float32)
    y = ops.gemm_i8(cu(a), cu(b), cu(sa), L.QI8_S_ROW, cu(sb), L.QI8_S_ROW, None, torch.bfloat16, act=L.QI8_ACT_GELU)
    pre = O.linear_w8a8_epilogue(O.int_mm(a, b), sa, sb.reshape(-1), None)
    ref = O.gelu_f32(O.round_bf16(pre))
    assert rel_fro(np_(y.float()), ref) < REL_BF16


def test_gemm_rejects_bad_shapes():
    a = torch.zeros(4, 24, dtype=torch.int8, device=dev())
    b = torch.zeros(16, 24, dtype=torch.int8, device=dev())
    with pytest.raises(AssertionError):
        ops.gemm_i8(a, b, out_dtype=torch.int32)  # K % 16 != 0


# ------------------------------------------------------ dequant / weights
def test_dequant_golden(golden):
    g = golden("triton_quant.npz")
    dw = ops.dequant(cu(g["qw"]), cu(g["sw"]), L.QI8_S_TILE128, 128, torch.float32)
    assert np.array_equal(np_(dw), g["dw"])
    da = ops.dequant(cu(g["y2"]), cu(g["s2"]), L.QI8_S_ROW_KBLOCK, 128, torch.float32)
    assert np.array_equal(np_(da), g["da2"])


def test_quant_weight_golden(golden):
    g = golden("triton_quant.npz")
    q, s = ops.quant_weight(cu(g["w"]), L.QI8_S_TILE128)
    assert np.array_equal(np_(q), g["qw"]) and np.array_equal(np_(s), g["sw"])
    g = golden("tensorwise.npz")
    q, s = ops.quant_weight(bf16_cu(g["w_bf16"]), L.QI8_S_SCALAR)
    assert np.array_equal(np_(q), g["q"]) and np.float32(np_(s)) == g["s"]


# -------------------------------------------------------- K4 converter
@pytest.mark.parametrize("tag,req,", [("row", L.QI8_REQ_ROW), ("glob", L.QI8_REQ_GLOBAL), ("block", L.QI8_REQ_BLOCK)])
def test_quip_convert_golden_pow2(golden, tag, req):
    g = golden("quip_convert.npz")
    q, s, deq = ops.quip_convert(cu(g["w"]), cu(g["s_u"]), cu(g["s_v"]), requant=req)
    assert np.array_equal(np_(q), g[f"{tag}_q"])
    assert np.array_equal(np_(s).reshape(g[f"{tag}_s"].shape), g[f"{tag}_s"])
    assert np.array_equal(np_(deq), g["row_deq"])


def test_quip_convert_golden_store_transformed(golden):
    g = golden("quip_convert.npz")
    q, s, deq = ops.quip_convert(cu(g["w"]), cu(g["s_u"]), cu(g["s_v"]), store_transformed=True)
    assert np.array_equal(np_(q), g["st_q"]) and np.array_equal(np_(s), g["st_s"])
    assert np.array_equal(np_(deq), g["st_deq"])


def test_quip_convert_golden_non_pow2(golden):
    g = golden("quip_convert.npz")
    w, su, sv = g["np_w"], g["np_s_u"], g["np_s_v"]
    q, s, deq = ops.quip_convert(cu(w), cu(su), cu(sv), requant=L.QI8_REQ_ROW)
    assert np.array_equal(np_(deq), g["np_deq"])
    assert np.array_equal(np_(q), g["np_q_row"]) and np.array_equal(np_(s), g["np_s_row"])
    qb, sb, _ = ops.quip_convert(cu(w), cu(su), cu(sv), requant=L.QI8_REQ_BLOCK, block=64)
    assert np.array_equal(np_(qb), g["np_q_block"]) and np.array_equal(np_(sb), g["np_s_block"])
    qt, st, _ = ops.quip_convert(cu(w), cu(su), cu(sv), store_transformed=True)
    assert np.array_equal(np_(qt), g["np_qrot"]) and np.array_equal(np_(st), g["np_srot"])


@pytest.mark.parametrize("M,N", [(3072, 1024), (1024, 3072), (1000, 700), (4096, 512), (600, 16384)])
def test_quip_convert_random_vs_oracle(M, N):
    r = rng(M + 3 * N)
    w = (r.standard_normal((M, N)) * 0.02).astype(np.float32)
    wb = torch.from_numpy(w).to(torch.bfloat16)
    Mp, Np = O.next_power_of_two(M), O.next_power_of_two(N)
    su = (r.integers(0, 2, Mp) * 2 - 1).astype(np.float32)
    sv = (r.integers(0, 2, Np) * 2 - 1).astype(np.float32)
    q, s, deq = ops.quip_convert(wb.to(dev()), cu(su), cu(sv), requant=L.QI8_REQ_BLOCK)
    qr, sr, dr = O.quip_convert(wb.float().numpy(), su, sv, "block", True)
    assert np.array_equal(np_(deq), dr)
    assert np.array_equal(np_(q), qr) and np.array_equal(np_(s).reshape(sr.shape), sr)


@pytest.mark.parametrize("M,N", [(128, 256), (96, 192), (1000, 700), (4096, 512), (300, 16384)])
def test_weight_rotate2d_vs_oracle(M, N):
    # the converter's incoherence rotation on its own, forward and inverse
    r = rng(7 * M + N)
    w = (r.standard_normal((M, N)) * 0.02).astype(np.float32)
    wb = torch.from_numpy(w).to(torch.bfloat16)
    Mp, Np = O.next_power_of_two(M), O.next_power_of_two(N)
    su = (r.integers(0, 2, Mp) * 2 - 1).astype(np.float32)
    sv = (r.integers(0, 2, Np) * 2 - 1).astype(np.float32)
    wr = ops.weight_rotate2d(wb.to(dev()), cu(su), cu(sv))
    ref = O.quip_rotate_weight(wb.float().numpy(), su, sv)
    assert np.array_equal(np_(wr), ref)
    back = ops.weight_rotate2d(wr, cu(su), cu(sv), inverse=True, shape=(M, N))
    assert np.array_equal(np_(back), O.quip_inverse_rotate(ref, su, sv, M, N))
    # orthogonal: the round trip returns the weight up to fp32 rounding
    assert np.max(np.abs(np_(back) - wb.float().numpy())) < 1e-6


def test_weight_rotate2d_rejects_bad_sizes():
    w = torch.zeros(8, 8, device=dev())
    with pytest.raises(AssertionError):
        ops.weight_rotate2d(w, torch.ones(12, device=dev()), torch.ones(8, device=dev()))  # 12 not a power of 2
    with pytest.raises(AssertionError):
        ops.weight_rotate2d(w, torch.ones(8, device=dev()), torch.ones(16, device=dev()), inverse=True)


# -------------------------------------------------- rotated W8A8 linear
def test_quip_w8a8_linear_vs_reference_fp32(golden):
    g = golden("quip_matmul.npz")
    x = cu(g["x"])
    xq, xs = ops.rotate_quant_rows(x, cu(g["s_v"]), 256)
    y_had = ops.gemm_i8(xq, cu(g["Q"]), xs, L.QI8_S_ROW, cu(g["scale"]), L.QI8_S_ROW, None, torch.float32)
    y = ops.unrotate_rows(y_had, cu(g["s_u"]), 128, None, torch.float32)
    assert rel_fro(np_(y), g["y"]) < 1e-2
    # and bit-exact against the oracle's W8A8 composition
    _, _, _, _, yo = O.quip_linear_w8a8(g["x"], g["Q"], g["scale"], g["s_u"], g["s_v"], 128, None)
    assert np.array_equal(np_(y), yo)
