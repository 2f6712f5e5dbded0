"""B200-native (sm_100a) QuIP W8A8 quantized-linear path for convert_to_quant.

Drop-in for the Triton kernels under ``convert_to_quant/comfy`` and the QuIP
converter's Hadamard path (ThunderFun/convert_to_quant_QuIP_INT8 v0.8.2),
backed by hand-written CUDA kernels in ``libqi8.so`` (C ABI: include/qi8.h).
"""

__version__ = "0.1.0"

from . import _lib  # noqa: F401
