"""Host utilities mirroring ``convert_to_quant/utils`` (float quantizers, Hadamard
transforms and the ``.comfy_quant`` metadata format)."""
