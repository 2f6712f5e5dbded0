"""GPU tests of the reference-facing operator surface: F.linear on
QuantizedTensor layouts, the kernel wrappers with the reference's signatures,
the QuIP converter class and the sharded linear, against the golden vectors
and the oracle."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle as O
from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import ops, sharding
from convert_to_quant_quip_int8_b200.comfy import hadamard_kernels as HK
from convert_to_quant_quip_int8_b200.comfy import int8_kernels as IK
from convert_to_quant_quip_int8_b200.comfy.int8_matmul_kernels import mm_8bit
from convert_to_quant_quip_int8_b200.comfy.quant_ops import QuantizedTensor, quip_hadamard_weight
from convert_to_quant_quip_int8_b200.converters.quip_int8 import HADAMARD_RTN, QuIPInt8Converter
from convert_to_quant_quip_int8_b200.utils import float_utils as FU

pytestmark = pytest.mark.gpu


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bf16_cu(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.fixture(autouse=True)
def _status():
    yield
    ops.device_status(reset=True)


@pytest.mark.parametrize("layout,name", [("TensorWiseINT8Layout", "tw"), ("AxisWiseINT8Layout", "aw")])
def test_flinear_tensor_axis_layouts_bitexact(golden, layout, name):
    g = golden("linear.npz")
    x, w, b = bf16_cu(g["x_bf16"]), bf16_cu(g["w_bf16"]), bf16_cu(g["bias_bf16"])
    wq = QuantizedTensor.from_float(w, layout)
    assert np.array_equal(wq._qdata.cpu().numpy(), g[f"{name}_wq"])
    assert np.array_equal(wq._layout_params["scale"].cpu().numpy(), g[f"{name}_ws"])
    y = F.linear(x, wq, b)
    assert y.dtype == torch.bfloat16 and y.shape == (33, 192)
    assert np.array_equal(bits(y), g[f"{name}_y_bf16"])
    # 3-D input keeps its batch shape
    y3 = F.linear(x.reshape(3, 11, 512), wq, b)
    assert np.array_equal(bits(y3.reshape(33, 192)), g[f"{name}_y_bf16"])


def test_quip_per_row_tensorwise_scale():
    # the QuIP default requant writes a per-row [N,1] scale under int8_tensorwise
    r = np.random.default_rng(1)
    x = torch.from_numpy(r.standard_normal((17, 256)).astype(np.float32)).to(torch.bfloat16)
    w = (torch.from_numpy(r.standard_normal((64, 256)).astype(np.float32)) * 0.02).cuda()
    q, s = ops.requant_weight(w, L.QI8_REQ_ROW)
    wq = QuantizedTensor(q, "TensorWiseINT8Layout", {"scale": s, "orig_dtype": torch.bfloat16})
    y = F.linear(x.cuda(), wq)
    _, _, _, yo = O.linear_w8a8(x.float().numpy(), q.cpu().numpy(), s.cpu().numpy().reshape(-1), None)
    assert np.array_equal(bits(y), O.f32_to_bf16(yo))


def test_blockwise_act_and_weight_layers(golden):
    g = golden("gemm_block.npz")
    x = bf16_cu(g["x_bf16"])
    wdeq = cu(O.weight_dequant(g["bq"], g["b_s"]))
    xa = QuantizedTensor.from_float(x, "BlockWiseINT8Layout", block_size=128, is_weight=False)
    assert np.array_equal(xa._qdata.cpu().numpy(), g["aq"])
    wq = QuantizedTensor(cu(g["bq"]), "BlockWiseINT8Layout",
                         {"scale": cu(g["b_s"]), "block_size": 128, "is_weight": True, "orig_dtype": torch.bfloat16})
    y = F.linear(xa, wq, cu(g["bias"]).to(torch.bfloat16))
    ref = O.int8_gemm_block(g["aq"], g["a_s"], g["bq"], g["b_s"], O.bf16_to_f32(O.f32_to_bf16(g["bias"])))
    assert y.dtype == torch.bfloat16 and rel(y.float().cpu().numpy(), ref) < 1e-2
    # dequantize path of the weight layout
    assert np.array_equal(wq.dequantize().float().cpu().numpy(), O.round_bf16(O.weight_dequant(g["bq"], g["b_s"])))
    del wdeq


def test_quip_block_weight_plain_input_w8a8():
    r = np.random.default_rng(2)
    x = torch.from_numpy(r.standard_normal((40, 512)).astype(np.float32)).to(torch.bfloat16)
    w = (torch.from_numpy(r.standard_normal((256, 512)).astype(np.float32)) * 0.02).cuda()
    q, s = ops.requant_weight(w, L.QI8_REQ_BLOCK)  # [256, 4, 1]
    wq = QuantizedTensor(q, "BlockWiseINT8Layout", {"scale": s, "block_size": 128, "is_weight": True,
                                                   "orig_dtype": torch.bfloat16})
    y = F.linear(x.cuda(), wq)
    xq, xs = O.quantize_int8_axiswise(x.float().numpy())
    ref = O.int8_gemm_block(xq, xs, q.cpu().numpy(), s.cpu().numpy().reshape(256, -1), None, b_layout="row")
    assert rel(y.float().cpu().numpy(), ref) < 1e-2


def test_quip_hadamard_layout_linear_bitexact():
    r = np.random.default_rng(3)
    M_out, K_in = 300, 700
    x = torch.from_numpy(r.standard_normal((21, K_in)).astype(np.float32)).to(torch.bfloat16)
    w = (torch.from_numpy(r.standard_normal((M_out, K_in)).astype(np.float32)) * 0.02).to(torch.bfloat16)
    bias = (torch.from_numpy(r.standard_normal(M_out).astype(np.float32)) * 0.01).to(torch.bfloat16)
    conv = QuIPInt8Converter(seed=5, store_transformed=True, **HADAMARD_RTN)
    q, s, deq, _, su, sv, hq, so, si = conv.convert(w.cuda())
    assert hq and (so, si) == (512, 1024) and q.shape == (512, 1024)
    wl = quip_hadamard_weight(q, s, su, sv, M_out, K_in)
    y = F.linear(x.cuda(), wl, bias.cuda())
    _, _, _, _, yo = O.quip_linear_w8a8(x.float().numpy(), q.cpu().numpy(), s.cpu().numpy().reshape(-1),
                                        su.cpu().numpy(), sv.cpu().numpy(), M_out, bias.float().numpy())
    assert np.array_equal(bits(y), O.f32_to_bf16(yo))
    # and close to the dense bf16 layer on the dequantized weight
    yd = x.float().numpy() @ deq.cpu().numpy().T + bias.float().numpy()
    assert rel(y.float().cpu().numpy(), yd) < 2e-2


@pytest.mark.parametrize("tag,kw", [("row", dict(requant_scheme="tensor")),
                                    ("glob", dict(requant_scheme="tensor", requant_tensor_use_per_row_scale=False)),
                                    ("block", dict(requant_scheme="block")), ("st", dict(store_transformed=True))])
def test_converter_class_matches_reference_golden(golden, tag, kw):
    g = golden("quip_convert.npz")
    conv = QuIPInt8Converter(seed=7, **HADAMARD_RTN, **kw)
    res = conv.convert(cu(g["w"]))
    assert np.array_equal(res[0].cpu().numpy(), g[f"{tag}_q"])
    assert np.array_equal(res[1].cpu().numpy().reshape(g[f"{tag}_s"].shape), g[f"{tag}_s"])
    assert tuple(res[1].shape) == tuple(g[f"{tag}_s"].shape)
    if tag == "st":
        # signs drawn exactly as the reference (CPU generator, s_u then s_v)
        assert np.array_equal(res[4].cpu().numpy(), g["s_u"]) and np.array_equal(res[5].cpu().numpy(), g["s_v"])
        assert (res[6], res[7], res[8]) == (True, 128, 256)
    else:
        assert res[4] is None and res[6] is False
    assert np.array_equal(res[2].cpu().numpy(), g["row_deq"] if tag != "st" else g["st_deq"])


def test_converter_rejects_unsupported_options():
    with pytest.raises(NotImplementedError):
        QuIPInt8Converter(use_learned_rounding=True)
    with pytest.raises(NotImplementedError):
        QuIPInt8Converter().convert(torch.zeros(16, 16, device="cuda"), activation_scales=torch.ones(16))


@pytest.mark.parametrize("tag", ["np", "p2"])
def test_converter_reference_defaults_golden(golden, tag):
    """The reference converter with its default arguments (act-order,
    diagonal rescaling, random permutation, damping, LDLQ), golden vectors
    from the reference itself."""
    g = golden("quip_convert_defaults.npz")
    res = QuIPInt8Converter(seed=7).convert(cu(g[f"{tag}_w"]))
    assert np.array_equal(res[0].cpu().numpy(), g[f"{tag}_q"])
    assert np.array_equal(res[1].cpu().numpy(), g[f"{tag}_s"])
    assert np.array_equal(res[2].cpu().numpy(), g[f"{tag}_deq"])


def test_kernel_wrappers_golden(golden):
    g = golden("triton_quant.npz")
    y, s = IK.act_quant(bf16_cu(g["x_bf16"]))
    assert np.array_equal(y.cpu().numpy(), g["y"]) and np.array_equal(s.cpu().numpy(), g["s"])
    qw, sw = IK.weight_quant(cu(g["w"]))
    assert np.array_equal(qw.cpu().numpy(), g["qw"]) and np.array_equal(sw.cpu().numpy(), g["sw"])
    assert np.array_equal(IK.weight_dequant(qw, sw, output_dtype=torch.float32).cpu().numpy(), g["dw"])
    assert np.array_equal(IK.act_dequant(cu(g["y2"]), cu(g["s2"]), output_dtype=torch.float32).cpu().numpy(), g["da2"])
    gm = golden("int_mm.npz")
    b_t = cu(gm["b"]).t()  # [K, N] view of the [N, K] weight, as mm_8bit receives w.t()
    assert np.array_equal(mm_8bit(cu(gm["a"]), b_t).cpu().numpy(), gm["c"])
    gb = golden("gemm_block.npz")
    c = IK.int8_addmm(cu(gb["aq"]), cu(gb["a_s"]), cu(gb["bq"]), cu(gb["b_s"]), cu(gb["bias"]))
    assert c.dtype == torch.float16
    ref = gb["c_fp16"].view(np.float16).astype(np.float32)
    assert rel(c.float().cpu().numpy(), ref) < 1e-3
    ga = golden("act_token.npz")
    q, s = FU.quantize_int8_axiswise(bf16_cu(ga["xa_bf16"]))
    assert np.array_equal(q.cpu().numpy(), ga["qa"]) and np.array_equal(s.cpu().numpy(), ga["sa"])
    gt = golden("tensorwise.npz")
    q, s = FU.quantize_int8_tensorwise(bf16_cu(gt["w_bf16"]))
    assert np.array_equal(q.cpu().numpy(), gt["q"]) and s.dim() == 0


def test_quip_int8_matmul_wrapper(golden):
    g = golden("quip_matmul.npz")
    y = IK.quip_int8_matmul(cu(g["x"]), cu(g["Q"]), cu(g["scale"]), cu(g["s_u"]), cu(g["s_v"]))
    assert y.dtype == torch.float32 and y.shape == (16, 128)
    assert rel(y.cpu().numpy(), g["y"]) < 1e-2


def test_hadamard_wrappers_golden(golden):
    g = golden("fwht.npz")
    assert np.array_equal(HK.fast_hadamard_transform(cu(g["x2"])).cpu().numpy(), g["y2"])
    assert np.array_equal(HK.fast_hadamard_transform_2d(cu(g["x5"])).cpu().numpy(), g["y5_2d"])
    y = HK.fast_hadamard_transform_with_signs(cu(g["x5"]), cu(g["s5r"]), cu(g["s5c"]))
    assert np.array_equal(y.cpu().numpy(), g["y5_2d_signs"])
    yi = HK.inverse_hadamard_transform_2d_with_signs(cu(g["x5"]), cu(g["s5r"]), cu(g["s5c"]), 60, 100)
    assert np.array_equal(yi.cpu().numpy(), g["y5_inv_2d_signs"])
    with pytest.raises(ValueError):
        HK.fast_hadamard_transform(torch.zeros(2, 12, device="cuda"))


@pytest.mark.parametrize("kind", ["row", "block"])
def test_column_sharded_linear_single_rank_equals_full(kind):
    r = np.random.default_rng(4)
    x = torch.from_numpy(r.standard_normal((32, 512)).astype(np.float32)).to(torch.bfloat16).cuda()
    w = (torch.from_numpy(r.standard_normal((256, 512)).astype(np.float32)) * 0.02).cuda()
    q, s = ops.requant_weight(w, L.QI8_REQ_ROW if kind == "row" else L.QI8_REQ_BLOCK)
    lin = sharding.ColumnShardedW8A8Linear(q, s, None, rank=0, world=1)
    y = lin(x)
    # two half-width shards computed separately and concatenated match the full layer
    halves = [sharding.ColumnShardedW8A8Linear(q, s, None, rank=rr, world=2).local(x) for rr in range(2)]
    assert torch.equal(torch.cat(halves, dim=1), y)


@pytest.mark.parametrize("kind", ["row", "block"])
def test_column_sharded_linear_overlapped_chunks(kind):
    # the chunked GEMM + asynchronous all-gather path over a one-rank NCCL group
    import torch.distributed as dist
    r = np.random.default_rng(6)
    x = torch.from_numpy(r.standard_normal((1000, 512)).astype(np.float32)).to(torch.bfloat16).cuda()
    w = (torch.from_numpy(r.standard_normal((512, 512)).astype(np.float32)) * 0.02).cuda()
    bias = torch.from_numpy(r.standard_normal(512).astype(np.float32)).to(torch.bfloat16).cuda()
    q, s = ops.requant_weight(w, L.QI8_REQ_ROW if kind == "row" else L.QI8_REQ_BLOCK)
    full = sharding.ColumnShardedW8A8Linear(q, s, bias, rank=0, world=1)(x)
    dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    try:
        lin = sharding.ColumnShardedW8A8Linear(q, s, bias, rank=0, world=1, chunks=4)
        assert lin.chunks == 4 and len(sharding.token_chunks(1000, 4)) == 4
        y = lin(x)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    assert torch.equal(y, full)


def test_conversion_partition_single_gpu():
    shapes = [(384, 256), (256, 640), (128, 128)]
    names = [f"t{i}" for i in range(3)]
    gens = [torch.Generator().manual_seed(i) for i in range(3)]
    make = lambda i: (torch.randn(*shapes[i], generator=gens[i]) * 0.02).to(torch.bfloat16)
    conv = QuIPInt8Converter(seed=0, requant_scheme="block", **HADAMARD_RTN)
    out = sharding.convert_partition(names, shapes, make, conv, rank=0, world=1,
                                     keep=lambda r: (r[0].cpu(), r[1].cpu()))
    assert sorted(out) == names
    assert out["t1"][0].shape == (256, 640) and out["t1"][1].shape == (256, 5, 1)
