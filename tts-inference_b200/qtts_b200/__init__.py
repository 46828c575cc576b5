"""qtts_b200 -- B200-native (sm_100a) quantized linears for the qtts Qwen3-TTS runtime.

The package mirrors the reference's quantization surface so it can stand in
for it:

* ``qtts_b200.quant`` -- ``apply_quantization``, ``build_method``,
  ``fp8_supported``, ``quantize_module`` and the method classes
  (reference: qtts/quant/__init__.py:3-5);
* ``qtts_b200.quant.kernels`` -- ``kernel_available`` and ``w8_gemm``
  (reference: qtts/quant/kernels.py:84-86, 138-177);
* ``qtts_b200.layers.linear`` -- ``LinearBase``, ``MergedLinear``,
  ``iter_linears`` (reference: qtts/layers/linear.py);
* ``qtts_b200.config.QuantConfig`` and its command-line flags
  (reference: qtts/config.py:50-98, 387-432).

The compute runs in ``lib/libqtts_b200.so`` (hand-written CUDA for sm_100a,
C ABI in ``include/qtts_b200.h``).
"""

__version__ = "0.1.0"
