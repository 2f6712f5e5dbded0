"""Checkpoint conversion driver (convert.py) against the checkpoint the
reference itself writes: ``convert_to_int8(..., optimizer="quip",
comfy_quant=True, no_learned_rounding=True)`` on a tiny model, in per-row
tensorwise, block and store-transformed modes (tests/golden/ckpt_quip.npz).

Pinned to the reference's file tensor for tensor: names, dtypes, shapes,
the int8 weights and scales (diagonal rescaling, random permutation,
damping and LDLQ as the reference's driver runs them, act-order off as the
fixture was made), the ``.comfy_quant`` JSON, the Hadamard flags and sizes,
the sign vectors and the tensors copied unchanged.  A two-rank run
(shards + merge) equals the one-rank file.
"""

import numpy as np
import pytest
import torch

from convert_to_quant_quip_int8_b200 import convert as C
from convert_to_quant_quip_int8_b200.utils import comfy_quant as CQ

pytestmark = pytest.mark.gpu

MODES = {"tw": {}, "blk": {"quip_requant_scheme": "block"}, "st": {"quip_store_transformed": True}}


def _tensors(g, prefix):
    out = {}
    for k, dt in zip(g[f"{prefix}__keys"], g[f"{prefix}__dtypes"]):
        a = g[f"{prefix}/{k}"]
        out[str(k)] = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) if dt == "bfloat16" else torch.from_numpy(a)
    return out


@pytest.fixture
def model_file(golden, tmp_path):
    from safetensors.torch import save_file
    g = golden("ckpt_quip.npz")
    path = tmp_path / "in.safetensors"
    save_file(_tensors(g, "in"), str(path))
    return g, path


@pytest.mark.parametrize("tag", list(MODES))
def test_checkpoint_matches_reference_layout(model_file, tmp_path, tag):
    from safetensors.torch import load_file
    g, src = model_file
    dst = tmp_path / f"out_{tag}.safetensors"
    C.convert_to_int8_quip(str(src), str(dst), quip_seed=7, quip_actorder=False, **MODES[tag])
    got = load_file(str(dst))
    ref = _tensors(g, tag)
    assert sorted(got) == sorted(ref)
    for k in ref:
        assert got[k].dtype == ref[k].dtype, k
        assert tuple(got[k].shape) == tuple(ref[k].shape), k
        assert torch.equal(got[k], ref[k]), k
    for base in ("blk.0.qkv", "blk.0.proj"):
        meta = CQ.tensor_to_dict(got[f"{base}.comfy_quant"])
        N = got[f"{base}.weight"].shape[1]
        scheme = "block" if tag == "blk" and N % 128 == 0 else "tensor"
        assert meta["format"] == ("int8_blockwise" if scheme == "block" else "int8_tensorwise")


def test_two_rank_shards_merge_to_the_one_rank_file(model_file, tmp_path):
    from safetensors import safe_open
    from safetensors.torch import load_file
    g, src = model_file
    one = tmp_path / "one.safetensors"
    C.convert_to_int8_quip(str(src), str(one), quip_seed=7, save_quant_metadata=True)
    two = tmp_path / "two.safetensors"
    stats = [C.convert_to_int8_quip(str(src), str(two), quip_seed=7, save_quant_metadata=True, rank=r, world=2)
             for r in range(2)]
    assert sorted(s["tensors"] for s in stats) == [1, 1]  # two weights, one per rank
    C.merge_shards(str(two), 2)
    a, b = load_file(str(one)), load_file(str(two))
    assert sorted(a) == sorted(b)
    for k in a:
        assert torch.equal(a[k], b[k]), k
    with safe_open(str(two), "pt") as f:
        layers = __import__("json").loads(f.metadata()["_quantization_metadata"])["layers"]
    assert sorted(layers) == ["blk.0.proj", "blk.0.qkv"]
