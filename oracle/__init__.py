"""CPU oracle for the quantized-linear path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference's algorithms for the path the
library accelerates, each function citing the reference file:line it follows.
It is the checker, never the thing measured or shipped: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it. Nothing under ``tts-inference_b200/`` imports it.

Parity pin: the restatement is checked against golden vectors produced by
running the reference's own Python code (``tests/golden/make_golden.py``
imports ``qtts`` from the reference checkout and records its outputs) on the
CPU; the quantizers also model torch's CUDA evaluation of ``tensor / number``
(``device="cuda"``, the default), pinned by the GPU tests against torch's own
GPU ops.
"""

from .qtts_ref import (  # noqa: F401
    bf16_round,
    div_by_number,
    e4m3_decode,
    e4m3_encode,
    float_steps,
    fp16_round,
    fp8_scaled_mm_reference,
    fp8_weight_only_reference,
    int8_w8a8_reference,
    naive_dequant_linear,
    round_to,
    quantize_act_fp8,
    quantize_act_int8,
    quantize_weight_fp8,
    quantize_weight_per_channel,
    rel_err,
    rms_norm_reference,
    silu_mul_reference,
    tune_quantize,
    w8a16_reference,
)
