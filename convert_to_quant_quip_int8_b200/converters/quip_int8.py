"""QuIP INT8 converter, Hadamard path (mirror of converters/quip_int8.py).

``QuIPInt8Converter(...).convert(weight)`` returns the reference's 9-tuple
``(q, scale, dequantized_weight, smooth_factors, s_u, s_v, hadamard_quip,
hadamard_size_out, hadamard_size_in)`` (converters/quip_int8.py:1031-1682).

What this converter computes (all in ``qi8_quip_convert`` on the GPU):
randomized two-sided Hadamard rotation with the reference's signs and
pad-to-power-of-two rule (:421-551), rotated-space per-row RTN with scale
``max(amax/127, 1e-12)`` (:1272-1274, 655) -- the reference's LDLQ with an
identity Hessian -- then the inverse rotation (:1452, 1489-1506) and either
``store_transformed`` output (:1558-1608) or the original-space requant
(:1614-1669).  For power-of-two shapes this is bit-identical to the
reference converter constructed with ``actorder=False,
use_diagonal_rescaling=False, use_random_permutation=False`` and ``H=None``.

The constructor keeps the reference's defaults (:33, :50, :52: act-order,
diagonal rescaling and random permutation all on).  With those on, the
reference's LDLQ error feedback is active even without calibration data
(the rescaled Hessian is no longer the identity) and about a fifth of the
int8 weights differ from the path above, so requesting them raises
``NotImplementedError`` instead of silently computing something else: pass
``actorder=False, use_diagonal_rescaling=False, use_random_permutation=False``.

Also outside this path (``NotImplementedError``): a calibrated Hessian,
learned rounding, greedy coordinate descent, SmoothQuant activation scales
and the non-Hadamard orthogonal rotation.  Streaming / memory options are
accepted and ignored (the whole weight lives in HBM).
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _lib as L
from .. import ops
from ..utils.hadamard import next_power_of_two

#: the keyword arguments that select the Hadamard/RTN path this converter implements
HADAMARD_RTN = dict(actorder=False, use_diagonal_rescaling=False, use_random_permutation=False)


class QuIPInt8Converter:
    def __init__(self, block_size: int = 128, percdamp: float = 0.01, device: str = "cuda", actorder: bool = True,
                 use_hadamard: bool = True, seed: Optional[int] = None, use_triton: bool = False,
                 lazy_updates: bool = True, use_learned_rounding: bool = False, ldlq_iterations: int = 1,
                 store_transformed: bool = False, streaming_mode: str = "balanced", streaming_thresholds=None,
                 no_memory_limits: bool = False, use_checkpointed_ldlq: bool = False,
                 checkpointed_ldlq_threshold: int = 8192, checkpoint_segments: int = 4,
                 requant_scheme: str = "tensor", requant_tensor_use_per_row_scale: bool = True,
                 use_diagonal_rescaling: bool = True, use_frobenius_scaling: bool = True,
                 use_random_permutation: bool = True, use_greedy_coordinate_descent: bool = False,
                 greedy_cd_iterations: int = 100, frobenius_rho: float = 1.0):
        unsupported = {"actorder": actorder, "use_diagonal_rescaling": use_diagonal_rescaling,
                       "use_random_permutation": use_random_permutation,
                       "use_learned_rounding": use_learned_rounding,
                       "use_greedy_coordinate_descent": use_greedy_coordinate_descent,
                       "use_hadamard=False": not use_hadamard}
        bad = [k for k, v in unsupported.items() if v]
        if bad:
            raise NotImplementedError(
                f"QuIP options outside the Hadamard/RTN path: {', '.join(bad)} (the reference enables act-order, "
                "diagonal rescaling and random permutation by default; pass actorder=False, "
                "use_diagonal_rescaling=False, use_random_permutation=False for the implemented path)")
        if requant_scheme not in ("tensor", "block"):
            raise ValueError(f"requant_scheme must be 'tensor' or 'block', got {requant_scheme!r}")
        self.block_size = block_size
        self.device = device
        self.seed = seed
        self.store_transformed = store_transformed
        self.requant_scheme = requant_scheme
        self.requant_tensor_use_per_row_scale = requant_tensor_use_per_row_scale
        self.use_hadamard = True
        self.low_memory = False
        self._workspace = None

    def _get_random_signs(self, n: int, generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """±1 fp32 signs (converters/quip_int8.py:236-242): CPU generator when seeded."""
        if generator is not None:
            return torch.randint(0, 2, (n,), device=generator.device, generator=generator).float() * 2 - 1
        return torch.randint(0, 2, (n,), device=self.device).float() * 2 - 1

    def signs(self, M: int, N: int):
        """``(s_u [M_pad], s_v [N_pad])`` in the reference's draw order (:524-530)."""
        gen = torch.Generator(device="cpu").manual_seed(self.seed) if self.seed is not None else None
        s_u = self._get_random_signs(next_power_of_two(M), gen)
        s_v = self._get_random_signs(next_power_of_two(N), gen)
        return s_u, s_v

    def _requant_code(self, N: int) -> int:
        if self.requant_scheme == "block" and N % self.block_size == 0:
            return L.QI8_REQ_BLOCK
        return L.QI8_REQ_ROW if self.requant_tensor_use_per_row_scale else L.QI8_REQ_GLOBAL

    def convert(self, weight: torch.Tensor, H: Optional[torch.Tensor] = None,
                activation_scales: Optional[torch.Tensor] = None, smoothquant_alpha: float = 0.5):
        if H is not None:
            raise NotImplementedError("a calibrated Hessian (LDLQ error feedback) is outside the Hadamard/RTN path")
        if activation_scales is not None:
            raise NotImplementedError("SmoothQuant activation scales are outside the Hadamard/RTN path")
        assert weight.dim() == 2, "weight must be 2-D"
        M, N = weight.shape
        s_u, s_v = self.signs(M, N)
        w = weight.to(self.device)
        if w.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            w = w.float()
        dev = w.device
        s_u, s_v = s_u.to(dev), s_v.to(dev)
        nbytes = ops.quip_workspace_bytes(M, N)
        if self._workspace is None or self._workspace.numel() < nbytes or self._workspace.device != dev:
            self._workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        q, scale, deq = ops.quip_convert(w, s_u, s_v, store_transformed=self.store_transformed,
                                         requant=self._requant_code(N), block=self.block_size,
                                         want_dequant=True, workspace=self._workspace)
        if self.store_transformed:
            return (q, scale, deq, None, s_u, s_v, True, next_power_of_two(M), next_power_of_two(N))
        return (q, scale, deq, None, None, None, False, 0, 0)

    def cleanup(self):
        self._workspace = None
