"""Linear stacks (Flux-shaped QuIP per-row, T5 axis-wise) on a reduced spec
list: the preallocated C-ABI forward, its CUDA-graph replay and the public
``F.linear(x, QuantizedTensor)`` path give identical bf16 outputs, and the
gather re-layout kernel matches its definition."""

import pytest
import torch
import torch.nn.functional as F

from convert_to_quant_quip_int8_b200 import ops
from convert_to_quant_quip_int8_b200.comfy.quant_ops import QuantizedTensor
from convert_to_quant_quip_int8_b200.stack import LinearSpec, LinearStack

pytestmark = pytest.mark.gpu


def _public_forward(st, layout):
    outs, kept = {}, {}
    for i, s in enumerate(st.specs):
        q, sc, b = st.weights[i]
        scale = sc.reshape(-1, 1) if layout == "TensorWiseINT8Layout" else sc
        w = QuantizedTensor(q, layout, {"scale": scale, "orig_dtype": torch.bfloat16})
        x = st.inputs[(s.tokens, s.k)] if s.src == "x" else F.gelu(kept[s.src])
        y = F.linear(x, w, b)
        kept[s.name] = y
        outs[s.name] = y
    return outs


@pytest.mark.parametrize("name", ["flux", "t5"])
def test_stack_forward_graph_and_public_api_agree(name):
    dev = torch.device("cuda", 0)
    specs = [LinearSpec("a.qkv", 300, 256, 768), LinearSpec("a.mlp0", 300, 256, 512),
             LinearSpec("a.mlp2", 300, 512, 256, "a.mlp0", True), LinearSpec("b.proj", 64, 512, 256)]
    st = LinearStack(name, dev, specs=specs)
    layout = "TensorWiseINT8Layout" if name == "flux" else "AxisWiseINT8Layout"
    ref = _public_forward(st, layout)
    got = {}
    for i, s in enumerate(st.specs):  # eager, one linear at a time (outputs share a scratch)
        st.run_linear(i, ops.L.stream_ptr(dev))
        got[s.name] = st.out_of[s.name].clone()
    for k in ref:
        assert torch.equal(got[k], ref[k]), k
    g = torch.cuda.CUDAGraph()
    st.forward()
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        st.forward()
    st.out_of["b.proj"].zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(st.out_of["b.proj"], ref["b.proj"])
    assert torch.equal(st.out_of["a.mlp0"], ref["a.mlp0"])
    del g


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.int8])
@pytest.mark.parametrize("world,T,n", [(2, 37, 24), (4, 5, 48), (3, 16, 7)])
def test_gather_layout_matches_definition(dtype, world, T, n):
    g = torch.arange(world * T * n, dtype=torch.float32).remainder(127).to(dtype).cuda().view(world * T, n)
    ld = world * n + 8
    out = torch.full((T, ld), -1, dtype=dtype, device="cuda")
    ops.gather_layout(g, world, out=out[:, : world * n])
    torch.cuda.synchronize()
    expect = g.view(world, T, n).permute(1, 0, 2).reshape(T, world * n)
    assert torch.equal(out[:, : world * n], expect)
    assert bool((out[:, world * n:] == -1).all())


def _oracle_linear(st, i, x_bf16, gelu=False):
    """The oracle's W8A8 linear (per-token int8, int32 GEMM, per-row weight
    scale, bias) on the stack's own weights; returns bf16 bits."""
    import numpy as np
    import oracle as O
    q, sc, b = st.weights[i]
    x = x_bf16.float().cpu().numpy()
    if gelu:
        x = O.round_bf16(O.gelu_f32(x))
    y = O.linear_w8a8(x, q.cpu().numpy(), sc.reshape(-1).cpu().numpy(),
                      None if b is None else b.float().cpu().numpy())[3]
    return O.f32_to_bf16(y).astype(np.uint16)


@pytest.mark.parametrize("name", ["flux", "t5"])
def test_stack_linears_match_oracle(name):
    """Every linear of a reduced stack, run by the graph-capturable C-ABI
    forward, equals the oracle's W8A8 linear bit for bit (the GELU-fed MLP
    down projection is checked on its quantized input instead, because CUDA's
    erff and the oracle's erf may differ in the last bit)."""
    import numpy as np
    dev = torch.device("cuda", 0)
    specs = [LinearSpec("a.qkv", 300, 256, 768), LinearSpec("a.mlp0", 300, 256, 512),
             LinearSpec("b.proj", 64, 512, 256)]
    st = LinearStack(name, dev, specs=specs)
    for i, s in enumerate(st.specs):
        st.run_linear(i, ops.L.stream_ptr(dev))
        got = st.out_of[s.name].cpu().view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(got, _oracle_linear(st, i, st.source(s))), s.name


def test_stack_token_split_rank_specs_and_rows():
    """Token split (full weights on every rank, 1/N of each linear's tokens):
    rank 0 of two gets half of every linear's tokens, the same weights as the
    single-rank stack, and on the same rows gives the same outputs."""
    dev = torch.device("cuda", 0)
    specs = [LinearSpec("a.qkv", 256, 256, 768), LinearSpec("a.mlp0", 256, 256, 512),
             LinearSpec("a.mlp2", 256, 512, 256, "a.mlp0", True), LinearSpec("b.proj", 64, 512, 256)]
    full = LinearStack("flux", dev, specs=specs)
    half = LinearStack("flux", dev, rank=0, world=2, shard="tokens", specs=specs)
    assert [s.tokens for s in half.specs] == [s.tokens // 2 for s in specs]
    assert not half.sharded
    for (qf, sf, bf), (qh, sh, bh) in zip(full.weights, half.weights):
        assert torch.equal(qf, qh) and torch.equal(sf, sh) and torch.equal(bf, bh)
    for key, x in half.inputs.items():
        x.copy_(full.inputs[(key[0] * 2, key[1])][: key[0]])
    sp = ops.L.stream_ptr(dev)
    for i, (sf_, sh_) in enumerate(zip(full.specs, half.specs)):
        full.run_linear(i, sp)
        half.run_linear(i, sp)
        assert torch.equal(half.out_of[sh_.name], full.out_of[sf_.name][: sh_.tokens]), sf_.name


def test_stack_lanes_overlap_equals_sequential():
    """Three lanes of a group (lanes 1 and 2 on their own streams, forked
    at the group's start and joined at its end): the overlapped forward,
    eager and replayed as a graph, writes the same bits as the linears run
    one at a time; a lane-0 linear after the join reads the lane-1 output."""
    dev = torch.device("cuda", 0)
    specs = [LinearSpec("g.img.mlp0", 200, 256, 512, lane=0, group="g"),
             LinearSpec("g.img.mlp2", 200, 512, 256, "g.img.mlp0", True, 0, "g"),
             LinearSpec("g.txt.mlp0", 64, 256, 512, lane=1, group="g"),
             LinearSpec("g.txt.mlp2", 64, 512, 256, "g.txt.mlp0", True, 1, "g"),
             LinearSpec("g.aux.proj", 96, 256, 192, lane=2, group="g"),
             LinearSpec("h.proj", 64, 256, 384, "g.txt.mlp2"),
             LinearSpec("h.out", 64, 384, 128, "h.proj"),
             LinearSpec("k.other", 200, 256, 128, "g.img.mlp2")]
    seq = LinearStack("flux", dev, specs=specs, overlap=False)
    sp = ops.L.stream_ptr(dev)
    ref = {}
    for i, s in enumerate(seq.specs):
        seq.run_linear(i, sp)
        ref[s.name] = seq.out_of[s.name].clone()
    ovl = LinearStack("flux", dev, specs=specs)
    assert ovl.overlap and sorted(ovl.sides) == [1, 2]
    assert [f for _, f in ovl.groups] == [True, False, False, False]
    for key, x in ovl.inputs.items():
        assert torch.equal(x, seq.inputs[key])
    ovl.forward()
    torch.cuda.synchronize()
    kept_or_last = ["g.img.mlp0", "g.img.mlp2", "g.txt.mlp0", "g.txt.mlp2", "g.aux.proj", "h.proj", "k.other"]
    for name in kept_or_last:
        assert torch.equal(ovl.out_of[name], ref[name]), name
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ovl.forward()
    for name in kept_or_last:
        ovl.out_of[name].zero_()
    g.replay()
    torch.cuda.synchronize()
    for name in kept_or_last:
        assert torch.equal(ovl.out_of[name], ref[name]), name
    del g
