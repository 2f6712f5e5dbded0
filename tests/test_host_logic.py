"""CPU tests of host-side logic: metadata format contract, sign generation,
scale-kind classification, error mapping, workload definitions."""

import numpy as np
import pytest
import torch

from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import ops
from convert_to_quant_quip_int8_b200.converters.quip_int8 import HADAMARD_RTN, QuIPInt8Converter
from convert_to_quant_quip_int8_b200.utils import comfy_quant as CQ
from convert_to_quant_quip_int8_b200.utils.hadamard import hadamard_matrix, next_power_of_two
from convert_to_quant_quip_int8_b200 import workloads as W
import oracle as O


def test_comfy_quant_tensor_roundtrip():
    t = CQ.create_comfy_quant_tensor("int8_blockwise", block_size=128)
    assert t.dtype == torch.uint8
    assert CQ.tensor_to_dict(t) == {"format": "int8_blockwise", "group_size": 128}
    t2 = CQ.create_comfy_quant_tensor("int8_tensorwise", block_size=128, full_precision_matrix_mult=True)
    assert CQ.tensor_to_dict(t2) == {"format": "int8_tensorwise", "full_precision_matrix_mult": True}
    with pytest.raises(ValueError):
        CQ.tensor_to_dict(torch.zeros(3, dtype=torch.int8))


def test_normalize_tensorwise_scales():
    ts = {"a.weight_scale": torch.tensor([0.5]), "a.weight": torch.zeros(2, 3).t(), "b.input_scale": torch.ones(2)}
    out, n = CQ.normalize_tensorwise_scales(ts)
    assert n == 1 and out["a.weight_scale"].dim() == 0 and out["a.weight"].is_contiguous()
    assert out["b.input_scale"].shape == (2,)


def test_quip_layer_tensor_names_and_dtypes():
    q = torch.zeros(512, 1024, dtype=torch.int8)
    s = torch.ones(512, 1)
    res = (q, s, None, None, torch.ones(512), -torch.ones(1024), True, 512, 1024)
    t = CQ.quip_layer_tensors("blk.attn", res)
    assert t["blk.attn.hadamard_quip"].dtype == torch.int8 and int(t["blk.attn.hadamard_quip"]) == 1
    assert t["blk.attn.hadamard_size_out"].dtype == torch.int32 and int(t["blk.attn.hadamard_size_in"]) == 1024
    assert t["blk.attn.sign_row"].dtype == torch.float32 and t["blk.attn.sign_col"].shape == (1024,)
    assert CQ.tensor_to_dict(t["blk.attn.comfy_quant"]) == {"format": "int8_tensorwise"}
    rb = (torch.zeros(64, 256, dtype=torch.int8), torch.ones(64, 2, 1), None, None, None, None, False, 0, 0)
    tb = CQ.quip_layer_tensors("mlp", rb)
    assert CQ.tensor_to_dict(tb["mlp.comfy_quant"]) == {"format": "int8_blockwise", "group_size": 128}
    assert "mlp.sign_row" not in tb


def test_converter_signs_match_reference(golden):
    g = golden("quip_convert.npz")
    s_u, s_v = QuIPInt8Converter(seed=7, **HADAMARD_RTN).signs(128, 256)
    assert np.array_equal(s_u.numpy(), g["s_u"]) and np.array_equal(s_v.numpy(), g["s_v"])
    su2, sv2 = QuIPInt8Converter(seed=7, **HADAMARD_RTN).signs(96, 192)
    assert np.array_equal(su2.numpy(), g["np_s_u"]) and np.array_equal(sv2.numpy(), g["np_s_v"])


def test_scale_kind_classification():
    assert ops.scale_kind(None, 8, 256, True) == L.QI8_S_NONE
    assert ops.scale_kind(torch.tensor(1.0), 8, 256, True) == L.QI8_S_SCALAR
    assert ops.scale_kind(torch.ones(8, 1), 8, 256, True) == L.QI8_S_ROW
    assert ops.scale_kind(torch.ones(8, 2, 1), 8, 256, True) == L.QI8_S_ROW_KBLOCK
    assert ops.scale_kind(torch.ones(2, 2), 256, 256, True) == L.QI8_S_TILE128
    with pytest.raises(AssertionError):
        ops.scale_kind(torch.ones(7), 8, 256, True)


def test_error_mapping():
    with pytest.raises(AssertionError):
        L.check(L.QI8_ESHAPE, "x")
    with pytest.raises(TypeError):
        L.check(L.QI8_EDTYPE, "x")
    with pytest.raises(L.QI8Error):
        L.check(L.QI8_ETIMEOUT, "x")
    L.check(L.QI8_OK)


def test_hadamard_matrix_and_pow2():
    h = hadamard_matrix(8)
    assert torch.allclose(h @ h.T, torch.eye(8), atol=1e-6)
    x = np.random.default_rng(0).standard_normal((3, 8)).astype(np.float32)
    assert np.allclose(O.fwht_rows(x), x @ h.numpy().T, atol=1e-6)
    assert [next_power_of_two(n) for n in (1, 3, 3072, 4096, 21504)] == [1, 4, 4096, 4096, 32768]


def test_workload_definitions():
    wl = W.DitMlpPair()
    assert wl.ops_per_step() == 2 * 2 * 4096 * 3072 * 12288
    su, sv = wl.w1_signs()
    assert su.shape == (16384,) and sv.shape == (4096,) and set(su.unique().tolist()) == {-1.0, 1.0}
    lin = W.flux_linears()
    assert len(lin) == 228
    ops_fwd = sum(2 * t * k * n for _, t, k, n in lin)
    assert abs(ops_fwd - 5.949e13) / 5.949e13 < 1e-3


def test_converter_rejects_options_on_cpu():
    for kw in (dict(use_learned_rounding=True), dict(use_greedy_coordinate_descent=True),
               dict(use_hadamard=False), dict(ldlq_iterations=2)):
        with pytest.raises(NotImplementedError):
            QuIPInt8Converter(**kw)
    with pytest.raises(ValueError):
        QuIPInt8Converter(requant_scheme="axis", **HADAMARD_RTN)


def test_converter_keeps_reference_defaults():
    """The reference turns act-order, diagonal rescaling and random
    permutation on by default (converters/quip_int8.py:33, 50, 52), and
    store_transformed turns rescaling off (:83-88)."""
    import inspect
    sig = inspect.signature(QuIPInt8Converter.__init__).parameters
    assert all(sig[k].default is True for k in HADAMARD_RTN)
    c = QuIPInt8Converter()
    assert c.actorder and c.use_diagonal_rescaling and c.use_random_permutation and c.percdamp == 0.01
    assert not QuIPInt8Converter(store_transformed=True).use_diagonal_rescaling


def test_conversion_driver_selects_2d_weights_and_names_shards():
    from convert_to_quant_quip_int8_b200 import convert as C
    shapes = {"a.weight": (8, 16), "a.bias": (8,), "norm.weight": (16,), "b.lora_A.weight": (4, 16),
              "c.weight": (32, 8), "emb": (10, 4)}
    assert C.weight_keys(shapes) == ["a.weight", "b.lora_A.weight", "c.weight"]
    assert C.weight_keys(shapes, exclude=lambda k: "lora" in k) == ["a.weight", "c.weight"]
    assert C.shard_path("/x/m.safetensors", 1, 4) == "/x/m.safetensors.rank1-of-4"


def test_stack_fork_groups():
    """The Flux stack forks each double block's txt linears onto lane 1
    (19 groups of 8, the single blocks alone); T5 runs q, k, v on lanes
    0, 1, 2 and wi_0, wi_1 on lanes 0, 1 of every layer; a token split
    keeps lanes and groups."""
    from convert_to_quant_quip_int8_b200.stack import LinearSpec, flux_specs, fork_groups, t5_specs
    fx = flux_specs()
    g = fork_groups(fx)
    forked = [ix for ix, f in g if f]
    assert len(forked) == 19 and all(len(ix) == 8 for ix in forked)
    assert len(g) == 19 + 76 and sum(len(ix) for ix, _ in g) == 228
    for ix in forked:
        names = [fx[i].name for i in ix]
        assert {fx[i].lane for i in ix if ".txt." in fx[i].name} == {1}
        assert {fx[i].lane for i in ix if ".img." in fx[i].name} == {0}
        assert len({n.split(".")[0] for n in names}) == 1
    # a consumer reads its producer on the same lane
    by_name = {s.name: s for s in fx}
    assert all(by_name[s.src].lane == s.lane for s in fx if s.src != "x")
    t5 = t5_specs()
    g5 = fork_groups(t5)
    assert sum(1 for _, f in g5 if f) == 48 and len(g5) == 24 * 4
    assert [t5[i].name.split(".")[1] for i in g5[0][0]] == ["q", "k", "v"]
    assert [t5[i].lane for i in g5[0][0]] == [0, 1, 2]
    # groups only join consecutive specs
    specs = [LinearSpec("a", 8, 16, 16, group="g"), LinearSpec("b", 8, 16, 16, lane=1, group="g"),
             LinearSpec("c", 8, 16, 16), LinearSpec("d", 8, 16, 16, lane=1, group="g")]
    assert fork_groups(specs) == [([0, 1], True), ([2], False), ([3], True)]
