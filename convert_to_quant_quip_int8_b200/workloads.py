"""Seeded synthetic workloads with the shapes of the QuIP W8A8 benchmarks.

All tensors are drawn on the CPU with ``torch.Generator('cpu').manual_seed``
in fp32 and cast to bf16 (so the CPU oracle sees identical inputs), then moved
to the GPU by the caller.  Signs follow the reference's draw order: one CPU
generator seeded with the layer seed, ``s_u`` (output dim) first, then
``s_v`` (converters/quip_int8.py:525-530).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch


def gen(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(seed)


def next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def quip_signs(seed: int, m_pad: int, n_pad: int) -> Tuple[torch.Tensor, torch.Tensor]:
    g = gen(seed)
    s_u = torch.randint(0, 2, (m_pad,), generator=g).float() * 2 - 1
    s_v = torch.randint(0, 2, (n_pad,), generator=g).float() * 2 - 1
    return s_u, s_v


def normal(shape, std: float, seed: int) -> torch.Tensor:
    return torch.randn(*shape, generator=gen(seed)) * std


def with_outliers(x: torch.Tensor, n_channels: int, factor: float, seed: int) -> torch.Tensor:
    idx = torch.randperm(x.shape[-1], generator=gen(seed))[:n_channels]
    x = x.clone()
    x[:, idx] *= factor
    return x


# ----------------------------------------------------------- DiT MLP pair
@dataclass
class DitMlpPair:
    """DiT MLP pair with block-128 (K) weight scales.

    x [4096, 3072] bf16 N(0,1) with 0.5% (15) outlier channels x30 (seeds 13/14);
    W1 [12288, 3072] N(0,0.02) seed 10, QuIP-rotated (signs seed 12) and
    requantized in original space with [12288, 24, 1] block scales;
    W2 [3072, 12288] N(0,0.02) seed 11, block-128 requantized (no rotation);
    exact-erf GELU between the projections.
    """
    tokens: int = 4096
    hidden: int = 3072
    ffn: int = 12288

    def activations(self) -> torch.Tensor:
        x = normal((self.tokens, self.hidden), 1.0, 13)
        n_out = max(1, round(0.005 * self.hidden))
        return with_outliers(x, n_out, 30.0, 14).to(torch.bfloat16)

    def w1(self) -> torch.Tensor:
        return normal((self.ffn, self.hidden), 0.02, 10).to(torch.bfloat16)

    def w2(self) -> torch.Tensor:
        return normal((self.hidden, self.ffn), 0.02, 11).to(torch.bfloat16)

    def w1_signs(self):
        return quip_signs(12, next_pow2(self.ffn), next_pow2(self.hidden))

    def ops_per_step(self, tokens: int = None) -> int:
        t = self.tokens if tokens is None else tokens
        return 2 * 2 * t * self.hidden * self.ffn


# ------------------------------------------------ single QuIP W8A8 linear
@dataclass
class SingleQuipLinear:
    """One QuIP tensorwise linear: W [4096, 4096] N(0,0.02) seed 0, signs seed 1,
    x [512, 4096] N(0,1) seed 2 with 40 outlier channels x20 (seed 3), bias
    N(0,0.01) seed 4."""
    tokens: int = 512
    dim: int = 4096

    def weight(self):
        return normal((self.dim, self.dim), 0.02, 0).to(torch.bfloat16)

    def signs(self):
        return quip_signs(1, next_pow2(self.dim), next_pow2(self.dim))

    def activations(self):
        return with_outliers(normal((self.tokens, self.dim), 1.0, 2), 40, 20.0, 3).to(torch.bfloat16)

    def bias(self):
        return normal((self.dim,), 0.01, 4).to(torch.bfloat16)


# ---------------------------------------------------- Flux-shaped stack
def flux_linears() -> List[Tuple[str, int, int, int]]:
    """(name, tokens, in_features, out_features) of the 228 linears of a
    Flux-shaped forward: 19 double-stream blocks (img T=4096, txt T=512) and 38
    single-stream blocks (T=4608)."""
    out = []
    for b in range(19):
        for stream, t in (("img", 4096), ("txt", 512)):
            out += [(f"double{b}.{stream}.qkv", t, 3072, 9216), (f"double{b}.{stream}.proj", t, 3072, 3072),
                    (f"double{b}.{stream}.mlp0", t, 3072, 12288), (f"double{b}.{stream}.mlp2", t, 12288, 3072)]
    for b in range(38):
        out += [(f"single{b}.linear1", 4608, 3072, 21504), (f"single{b}.linear2", 4608, 15360, 3072)]
    return out


def conversion_sweep_tensors() -> List[Tuple[str, int, int]]:
    """The 304 weight shapes of the whole-model conversion sweep: the Flux
    double-block tensors plus the single-block set taken twice."""
    out = []
    for b in range(19):
        for stream in ("img", "txt"):
            out += [(f"double{b}.{stream}.qkv", 9216, 3072), (f"double{b}.{stream}.proj", 3072, 3072),
                    (f"double{b}.{stream}.mlp0", 12288, 3072), (f"double{b}.{stream}.mlp2", 3072, 12288)]
    for rep in range(2):
        for b in range(38):
            out += [(f"single{b}.{rep}.linear1", 21504, 3072), (f"single{b}.{rep}.linear2", 3072, 15360)]
    return out


# ---------------------------------------------------- T5-XXL encoder stack
def ldlq_block_tensors() -> List[Tuple[str, int, int]]:
    """The weights of one Flux double-stream block (img and txt: qkv, proj,
    mlp0, mlp2) and one single-stream block (linear1, linear2): 10 tensors,
    ``(name, out, in)``, for the converter with the reference's defaults."""
    return [t for t in conversion_sweep_tensors() if t[0].startswith(("double0.", "single0.0."))]


def t5_linears() -> List[Tuple[str, int, int, int]]:
    """(name, tokens, in_features, out_features) of the 168 linears of a
    T5-XXL-shaped encoder forward (d_model 4096, d_ff 10240, 24 layers,
    batch 8 x 512 tokens): q, k, v, o 4096->4096, gated-GELU wi_0 / wi_1
    4096->10240 and wo 10240->4096."""
    t = 8 * 512
    out = []
    for layer in range(24):
        pre = f"encoder{layer}"
        out += [(f"{pre}.q", t, 4096, 4096), (f"{pre}.k", t, 4096, 4096), (f"{pre}.v", t, 4096, 4096),
                (f"{pre}.o", t, 4096, 4096), (f"{pre}.wi_0", t, 4096, 10240), (f"{pre}.wi_1", t, 4096, 10240),
                (f"{pre}.wo", t, 10240, 4096)]
    return out


def student_t_outliers(x: torch.Tensor, frac: float, nu: int, seed: int) -> torch.Tensor:
    """Replaces ``frac`` of the channels of ``x`` [T, C] by Student-t(nu)
    samples (heavy-tailed outlier channels), seeded on the CPU."""
    g = gen(seed)
    n_ch = max(1, round(frac * x.shape[-1]))
    idx = torch.randperm(x.shape[-1], generator=g)[:n_ch]
    # Student-t(nu) = N(0,1) / sqrt(chi2(nu) / nu); chi2 of integer nu = sum of nu squared N(0,1)
    z = torch.randn(x.shape[0], n_ch, generator=g)
    chi2 = (torch.randn(int(nu), x.shape[0], n_ch, generator=g) ** 2).sum(0)
    x = x.clone()
    x[:, idx] = (z / torch.sqrt(chi2 / nu)).to(x.dtype)
    return x
