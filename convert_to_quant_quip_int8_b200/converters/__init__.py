"""Converters: the QuIP INT8 converter's Hadamard path on libqi8."""
