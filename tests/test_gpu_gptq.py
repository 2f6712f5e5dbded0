"""GPU parity of the GPTQ / LDLQ block kernel (comfy/gptq_kernels.py:11-124)
against the reference's own kernel executed by the Triton interpreter
(tests/golden/gptq_block.npz) and against the oracle at the converter's
block size: int8 codes, errors and the updated weight block bit-exact."""

import numpy as np
import pytest
import torch

import oracle as O
from convert_to_quant_quip_int8_b200 import ops
from convert_to_quant_quip_int8_b200.comfy import gptq_kernels as GK

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    ops.device_status(reset=True)


def test_gptq_block_golden(golden):
    g = golden("gptq_block.npz")
    for tag in ("row", "scalar"):
        W = torch.from_numpy(g["w"]).cuda()
        Q, E = GK.triton_gptq_quant_block(W, torch.from_numpy(g["hinv"]).cuda(),
                                          torch.from_numpy(g[f"{tag}_scale"]).cuda())
        assert np.array_equal(Q.cpu().numpy(), g[f"{tag}_q"])
        assert np.array_equal(E.cpu().numpy(), g[f"{tag}_err"])
        assert np.array_equal(W.cpu().numpy(), g[f"{tag}_w_out"])  # updated in place


@pytest.mark.parametrize("M,B", [(1, 128), (300, 128), (4096, 128), (1000, 37)])
def test_gptq_block_vs_oracle(M, B):
    r = np.random.default_rng(M + B)
    w = (r.standard_normal((M, B)) * 0.02).astype(np.float32)
    x = r.standard_normal((4 * B, B)).astype(np.float32)
    h = x.T @ x / (4 * B) + 0.01 * np.eye(B, dtype=np.float32)
    hinv = np.linalg.cholesky(np.linalg.inv(h)).T.astype(np.float32)  # upper Cholesky factor of H^-1
    sc = np.maximum(np.abs(w).max(axis=1, keepdims=True) / 127, 1e-8).astype(np.float32)
    W = torch.from_numpy(w).cuda()
    Q, E = GK.triton_gptq_quant_block(W, torch.from_numpy(hinv).cuda(), torch.from_numpy(sc).cuda())
    q_ref, e_ref, w_ref = O.gptq_quant_block(w, hinv, sc)
    assert np.array_equal(Q.cpu().numpy(), q_ref)
    assert np.array_equal(E.cpu().numpy(), e_ref)
    assert np.array_equal(W.cpu().numpy(), w_ref)


def test_gptq_block_strided_view_left_unchanged_like_the_reference():
    base = torch.randn(64, 256, device="cuda") * 0.02
    view = base[:, 64:192]
    before = view.clone()
    hinv = torch.eye(128, device="cuda")
    Q, E = GK.triton_gptq_quant_block(view, hinv, torch.full((64, 1), 1e-3, device="cuda"))
    assert torch.equal(view, before)  # the reference updates a contiguous copy
    assert Q.shape == (64, 128) and E.dtype == torch.float32
