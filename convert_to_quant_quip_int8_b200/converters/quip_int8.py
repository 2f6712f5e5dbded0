"""QuIP INT8 converter, Hadamard path (mirror of converters/quip_int8.py).

``QuIPInt8Converter(...).convert(weight, H=None)`` returns the reference's
9-tuple ``(q, scale, dequantized_weight, smooth_factors, s_u, s_v,
hadamard_quip, hadamard_size_out, hadamard_size_in)``
(converters/quip_int8.py:1031-1682), with the reference's defaults:

* diagonal rescaling ``D = clamp((diag H / colsumsq W) ** 0.25, 0.1, 10)``
  (:244-287; off when ``store_transformed``, :83-88),
* the randomized two-sided Hadamard rotation of W and H with the
  reference's signs and pad-to-power-of-two rule (:421-551),
* the random column permutation drawn after the signs (:306-352, 610-612),
* dead-column handling, damping ``percdamp * mean(diag H)`` and the
  act-order permutation (:1105-1146),
* the fp64 factorization of the damped Hessian to the upper Cholesky factor
  of its inverse (:1195-1216, identity on a non-positive pivot),
* the blocked lazy LDLQ pass with per-row scales (:813-945, 638-672,
  1272-1274),
* then act-order / permutation undone, the inverse rotation, ``W / D``
  (:1348-1513) and either the ``store_transformed`` output (:1558-1608) or
  the original-space requant (:1614-1669).

Device work runs in libqi8 (``qi8_col_sumsq``, ``qi8_scale2d``,
``qi8_weight_rotate2d``, ``qi8_ldlq_prepare``, ``qi8_hinv_upper``,
``qi8_ldlq``, ``qi8_ldlq_finish``, ``qi8_requant_weight``); the host
computes the O(N) vectors in between with the reference's own torch CPU
calls: D from the column sums, the random permutation from the seeded CPU
generator, the damping mean and the act-order ``argsort`` (whose tie order
is that of torch's unstable CPU sort, so it is part of the output).

With ``H=None``, no diagonal rescaling and a power-of-two input width the
rotated Hessian is exactly diagonal (each Hadamard row's butterflies stay
in {0, +-2^s c}), so LDLQ reduces to per-row RTN in any column order and the
single-kernel ``qi8_quip_convert`` path computes the same result.

Outside this path (``NotImplementedError``): learned rounding, greedy
coordinate descent, SmoothQuant activation scales, the non-Hadamard
orthogonal rotation and more than one LDLQ iteration.  Streaming / memory
options are accepted and ignored (the whole weight lives in HBM).  The
reference's LDLQ runs its cross-block updates under bf16 autocast on a CUDA
device and routes N >= 8192 through ``checkpointed_ldlq`` on CPU-only
hosts; this converter computes the fp32 single-pass arithmetic at every size.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _lib as L
from .. import ops
from ..utils.hadamard import next_power_of_two

#: keyword arguments that turn off the QuIP options with extra passes
#: (act-order, diagonal rescaling, random permutation)
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
        unsupported = {"use_learned_rounding": use_learned_rounding,
                       "use_greedy_coordinate_descent": use_greedy_coordinate_descent,
                       "use_hadamard=False": not use_hadamard,
                       f"ldlq_iterations={ldlq_iterations}": ldlq_iterations != 1}
        bad = [k for k, v in unsupported.items() if v]
        if bad:
            raise NotImplementedError(f"QuIP options outside the Hadamard LDLQ path: {', '.join(bad)}")
        if requant_scheme not in ("tensor", "block"):
            raise ValueError(f"requant_scheme must be 'tensor' or 'block', got {requant_scheme!r}")
        self.block_size = block_size
        self.percdamp = percdamp
        self.device = device
        self.seed = seed
        self.actorder = actorder
        self.store_transformed = store_transformed
        self.requant_scheme = requant_scheme
        self.requant_tensor_use_per_row_scale = requant_tensor_use_per_row_scale
        # store_transformed keeps no D_tilde, so the reference turns rescaling off (:83-88)
        self.use_diagonal_rescaling = use_diagonal_rescaling and not store_transformed
        self.use_random_permutation = use_random_permutation
        self.use_hadamard = True
        self.low_memory = False
        self._workspace = None

    def _get_random_signs(self, n: int, generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """±1 fp32 signs (converters/quip_int8.py:236-242): CPU generator when seeded."""
        if generator is not None:
            return torch.randint(0, 2, (n,), device=generator.device, generator=generator).float() * 2 - 1
        return torch.randint(0, 2, (n,), device=self.device).float() * 2 - 1

    def _generator(self):
        return torch.Generator(device="cpu").manual_seed(self.seed) if self.seed is not None else None

    def signs(self, M: int, N: int, gen=None):
        """``(s_u [M_pad], s_v [N_pad])`` in the reference's draw order (:524-530)."""
        gen = self._generator() if gen is None else gen
        s_u = self._get_random_signs(next_power_of_two(M), gen)
        s_v = self._get_random_signs(next_power_of_two(N), gen)
        return s_u, s_v

    def _requant_code(self, N: int) -> int:
        if self.requant_scheme == "block" and N % self.block_size == 0:
            return L.QI8_REQ_BLOCK
        return L.QI8_REQ_ROW if self.requant_tensor_use_per_row_scale else L.QI8_REQ_GLOBAL

    def convert(self, weight: torch.Tensor, H: Optional[torch.Tensor] = None,
                activation_scales: Optional[torch.Tensor] = None, smoothquant_alpha: float = 0.5):
        if activation_scales is not None:
            raise NotImplementedError("SmoothQuant activation scales are outside the Hadamard LDLQ path")
        assert weight.dim() == 2, "weight must be 2-D"
        M, N = weight.shape
        if H is None and not self.use_diagonal_rescaling and N == next_power_of_two(N):
            return self._convert_rtn(weight)
        return self._convert_ldlq(weight, H)

    def _convert_rtn(self, weight: torch.Tensor):
        """Identity Hessian, no rescaling, power-of-two width: one fused kernel."""
        M, N = weight.shape
        gen = self._generator()
        s_u, s_v = self.signs(M, N, gen)
        if self.use_random_permutation:  # consume the reference's draw; RTN is column-order invariant
            torch.randperm(next_power_of_two(N), device="cpu", generator=gen)
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

    def _convert_ldlq(self, weight: torch.Tensor, H: Optional[torch.Tensor]):
        """The reference's full QuIP pass (:1031-1669) on the GPU."""
        if not (16 <= self.block_size <= 128 and self.block_size % 16 == 0):
            raise NotImplementedError(f"LDLQ block_size {self.block_size} (16..128, a multiple of 16, supported)")
        M, N = weight.shape
        Mp, Np = next_power_of_two(M), next_power_of_two(N)
        if Mp > 32768 or Np > 32768:
            raise ValueError(f"padded weight {Mp}x{Np} exceeds 32768 in a dimension")
        W = weight.to(self.device, dtype=torch.float32).contiguous()
        dev = W.device
        L.require_cuda(W)
        Hd = None
        if H is not None:
            assert tuple(H.shape) == (N, N), f"H must be [{N}, {N}]"
            Hd = H.to(dev, dtype=torch.float32).contiguous()
        gen = self._generator()
        # diagonal rescaling (:244-287): O(N) vector math on the host, as the reference computes it
        D = Dd = None
        if self.use_diagonal_rescaling:
            wtw = ops.col_sumsq(W).cpu()
            hdiag = torch.ones(N, dtype=torch.float32) if Hd is None else torch.diagonal(Hd).cpu()
            ratio = hdiag.clamp(min=1e-12).double() / wtw.clamp(min=1e-12).double()
            D = torch.pow(ratio, 0.25).to(torch.float32).clamp(min=0.1, max=10.0)
            Dd = D.to(dev)
            Dinv = (1.0 / D).to(dev)
            Wr = ops.scale2d(W, (M, N), col=Dd)
            Hr = ops.scale2d(Hd, (N, N), row=Dinv, col=Dinv, device=dev)
        else:
            Wr = W
            Hr = Hd if Hd is not None else ops.scale2d(None, (N, N), device=dev)
        # incoherence rotation (:523-551) and random permutation (:336-340)
        s_u, s_v = self.signs(M, N, gen)
        s_u, s_v = s_u.to(dev), s_v.to(dev)
        Wrot = ops.weight_rotate2d(Wr, s_u, s_v)
        Hrot = ops.weight_rotate2d(Hr, s_v, s_v)
        del Wr, Hr
        if self.use_random_permutation:
            perm = torch.randperm(Np, device="cpu", generator=gen) if gen is not None else torch.randperm(Np)
        else:
            perm = torch.arange(Np)
        # dead columns, damping, act-order (:1105-1146) on the N-vector diagonal
        hdiag = torch.diagonal(Hrot).cpu()[perm]
        dead = hdiag == 0
        damp = self.percdamp * torch.mean(hdiag.double()).float()
        hkey = torch.where(dead, torch.ones_like(hdiag), hdiag) + damp
        order = torch.argsort(hkey, descending=True) if self.actorder else torch.arange(Np)
        cols = perm[order].to(torch.int32).to(dev)
        Wp, scale, Hrev = ops.ldlq_prepare(Wrot, Hrot, cols, dead[order].to(torch.uint8).to(dev),
                                           hkey[order].to(dev))
        del Wrot, Hrot
        Hinv, info = ops.hinv_upper(Hrev)
        del Hrev
        if int(info.item()) != 0:  # not positive definite: the reference falls back to the identity
            Hinv = ops.eye_f32(Np, dev)
        Q = ops.ldlq(Wp, Hinv, scale, self.block_size)
        del Wp, Hinv
        deq_t, q_st = ops.ldlq_finish(Q, scale, cols, want_deq=True, want_q=self.store_transformed)
        deq = ops.weight_rotate2d(deq_t, s_u, s_v, inverse=True, shape=(M, N))
        del deq_t
        if Dd is not None:
            deq = ops.scale2d(deq, (M, N), col=Dd, divide=True)
        if self.store_transformed:
            return (q_st, scale, deq, None, s_u, s_v, True, Mp, Np)
        q, s = ops.requant_weight(deq, self._requant_code(N), self.block_size)
        return (q, s, deq, None, None, None, False, 0, 0)

    def cleanup(self):
        self._workspace = None
