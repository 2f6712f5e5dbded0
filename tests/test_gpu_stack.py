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
