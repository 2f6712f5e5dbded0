"""CPU-side checks of the C ABI library: it loads and exports every symbol
that include/qi8.h declares, with no GPU present."""

import ctypes
import os
import re

import pytest

from convert_to_quant_quip_int8_b200 import _lib as L
from convert_to_quant_quip_int8_b200 import build as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qi8.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qi8_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    B.build()
    return L.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("qi8_rotate_quant_rows", "qi8_gemm_i8", "qi8_unrotate_rows", "qi8_quip_convert"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} not exported by libqi8.so"


def test_binding_table_matches_header():
    assert sorted(L.SIGNATURES) == declared_symbols()


def test_version_and_no_device(lib):
    assert lib.qi8_version() == 1
    # no GPU in this container: the device query reports "unsupported" instead of crashing
    assert lib.qi8_device_supported(0) == 0


def test_calls_fail_loudly_without_device(lib):
    rc = lib.qi8_gemm_i8(None, None, 1, 16, 16, None, 0, None, 0, None, 0, None, 0, 16, 0, None)
    assert rc == L.QI8_EUNSUPPORTED
    assert "sm_100" in L.last_error()


def test_wrappers_reject_cpu_tensors():
    import torch
    from convert_to_quant_quip_int8_b200 import ops
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quant_rows(torch.zeros(2, 16))
