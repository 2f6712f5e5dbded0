"""ComfyUI-compatible INT8 operator surface (mirror of ``convert_to_quant/comfy``).

``quant_ops``            QuantizedTensor, layouts, aten handlers
``int8_kernels``         act/weight (de)quant, block-scaled GEMMs, QuIP matmul
``int8_matmul_kernels``  ``mm_8bit`` (int8 x int8 -> int32)
``hadamard_kernels``     fast Walsh-Hadamard transforms
All compute runs in libqi8 (sm_100a); there is no CPU path.
"""

__all__ = ["quant_ops", "int8_kernels", "int8_matmul_kernels", "hadamard_kernels"]
