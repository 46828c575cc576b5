"""Quantization: one hook on ``LinearBase``, applied after the weights load.

Same public surface as the reference (qtts/quant/__init__.py:3-5).
"""

from .base import apply_quantization, build_method, fp8_supported, quantize_module

__all__ = ["apply_quantization", "build_method", "fp8_supported", "quantize_module"]
