"""Checkpoint conversion driver: a safetensors model in, a ComfyUI INT8
safetensors checkpoint out, with the QuIP Hadamard path on the GPU.

This is the QuIP branch of the reference's ``convert_to_int8``
(quantization.py:100-787) restricted to what this package implements:

* weight selection: every 2-D tensor whose key ends in ``.weight``
  (quantization.py:364-372), minus an optional exclusion predicate;
* per weight: ``QuIPInt8Converter(...).convert`` constructed as the
  reference's driver constructs it (quantization.py:590-607: act-order from
  ``quip_actorder``, diagonal rescaling and random permutation at their
  defaults, ``H=None`` without calibration data; signs and permutation
  seeded by ``quip_seed`` and drawn on the CPU exactly as the reference),
  then the per-layer tensors with the reference's names and dtypes
  (quantization.py:651-727): ``weight`` int8, ``weight_scale`` fp32,
  ``comfy_quant`` uint8 JSON, and in store-transformed mode
  ``hadamard_quip`` / ``hadamard_size_out`` / ``hadamard_size_in`` /
  ``sign_row`` / ``sign_col``;
* every other tensor is copied unchanged (quantization.py:762-765);
* 1-element scales are saved 0-d (``normalize_tensorwise_scales``,
  quantization.py:778-783) and ``_quantization_metadata`` is added on
  request (:773-776).

Calibration data, SmoothQuant, learned rounding, LoRA merging and the
reference's other optimizers are not part of this path (the reference's
``--simple`` QuIP conversion: no bias correction from synthetic
calibration data).

Multi-GPU: weights are independent units.  ``rank`` of ``world`` converts its
longest-processing-time share (``sharding.plan_partition`` on the padded
size, the same plan on every rank, no collective on the data path) and writes
a shard file; ``merge_shards`` assembles the checkpoint once every shard
exists.  While the GPU converts one weight, a host thread reads and pins the
next one.
"""

from __future__ import annotations

import concurrent.futures
import json
import os
import time
from typing import Callable, Dict, List, Optional

import torch

from .converters.quip_int8 import QuIPInt8Converter
from .sharding import plan_partition
from .utils import comfy_quant as CQ


def weight_keys(names_and_shapes: Dict[str, tuple], exclude: Optional[Callable[[str], bool]] = None) -> List[str]:
    """The 2-D ``.weight`` tensors the reference's driver quantizes, sorted."""
    keys = [k for k, shp in names_and_shapes.items() if k.endswith(".weight") and len(shp) == 2]
    if exclude is not None:
        keys = [k for k in keys if not exclude(k)]
    return sorted(keys)


def shard_path(output_file: str, rank: int, world: int) -> str:
    return f"{output_file}.rank{rank}-of-{world}"


def convert_to_int8_quip(input_file: str, output_file: str, *, comfy_quant: bool = True,
                         quip_seed: Optional[int] = None, quip_actorder: bool = True,
                         quip_store_transformed: bool = False,
                         quip_requant_scheme: str = "tensor", quip_requant_tensor_per_row: bool = True,
                         block_size: int = 128, save_quant_metadata: bool = False, device: Optional[str] = None,
                         rank: int = 0, world: int = 1, exclude: Optional[Callable[[str], bool]] = None) -> dict:
    """Converts ``input_file`` and writes ``output_file`` (``world == 1``) or this
    rank's shard (``world > 1``; call :func:`merge_shards` afterwards).
    Returns ``{"tensors", "params", "seconds", "path"}`` for this rank."""
    from safetensors import safe_open
    from safetensors.torch import save_file

    if not comfy_quant:
        raise NotImplementedError("only the comfy_quant checkpoint layout is produced")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    t0 = time.perf_counter()
    with safe_open(input_file, framework="pt", device="cpu") as f:
        names = list(f.keys())
        shapes = {k: tuple(f.get_slice(k).get_shape()) for k in names}
        metadata = f.metadata() or {}
        wkeys = weight_keys(shapes, exclude)
        plan = plan_partition([shapes[k] for k in wkeys], world)[rank]
        mine = [wkeys[i] for i in plan]
        conv = QuIPInt8Converter(block_size=block_size, device=str(dev), seed=quip_seed, actorder=quip_actorder,
                                 store_transformed=quip_store_transformed, requant_scheme=quip_requant_scheme,
                                 requant_tensor_use_per_row_scale=quip_requant_tensor_per_row)

        def read(key):
            return f.get_tensor(key).pin_memory()

        out: Dict[str, torch.Tensor] = {}
        layers = {}
        params = 0
        with concurrent.futures.ThreadPoolExecutor(max_workers=1) as pool:
            nxt = pool.submit(read, mine[0]) if mine else None
            for i, key in enumerate(mine):
                w_host = nxt.result()
                nxt = pool.submit(read, mine[i + 1]) if i + 1 < len(mine) else None
                w = w_host.to(dev, non_blocking=True)
                base = key[: -len(".weight")]
                res = conv.convert(w)
                t = CQ.quip_layer_tensors(base, res, block_size)
                out.update(t)
                meta = CQ.tensor_to_dict(t[f"{base}.comfy_quant"])
                layers[base] = meta
                params += w.numel()
        if rank == 0:
            # tensors that are not quantized travel unchanged
            for k in names:
                if k not in wkeys:
                    out[k] = f.get_tensor(k)
    torch.cuda.synchronize(dev)
    out, _ = CQ.normalize_tensorwise_scales(out)
    save_meta = dict(metadata)
    if save_quant_metadata and layers:
        save_meta["_quantization_metadata"] = json.dumps({"format_version": "1.0", "layers": layers})
    path = output_file if world == 1 else shard_path(output_file, rank, world)
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    save_file(out, path, metadata={k: str(v) for k, v in save_meta.items()} or None)
    return {"tensors": len(mine), "params": params, "seconds": time.perf_counter() - t0, "path": path}


def merge_shards(output_file: str, world: int, remove: bool = True) -> str:
    """Assembles the per-rank shards of :func:`convert_to_int8_quip` into
    ``output_file`` (the union of their tensors; rank 0's metadata, with the
    layers of every shard in ``_quantization_metadata`` when present)."""
    from safetensors import safe_open
    from safetensors.torch import save_file

    tensors: Dict[str, torch.Tensor] = {}
    meta: Dict[str, str] = {}
    layers = {}
    for r in range(world):
        p = shard_path(output_file, r, world)
        with safe_open(p, framework="pt", device="cpu") as f:
            m = f.metadata() or {}
            if r == 0:
                meta = dict(m)
            if "_quantization_metadata" in m:
                layers.update(json.loads(m["_quantization_metadata"])["layers"])
            for k in f.keys():
                tensors[k] = f.get_tensor(k)
    if layers:
        meta["_quantization_metadata"] = json.dumps({"format_version": "1.0", "layers": layers})
    save_file(tensors, output_file, metadata=meta or None)
    if remove:
        for r in range(world):
            os.remove(shard_path(output_file, r, world))
    return output_file
