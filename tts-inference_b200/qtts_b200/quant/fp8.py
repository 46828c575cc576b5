"""fp8 (e4m3) quantization methods.

:class:`Fp8Method` keeps the reference's W8A8 contract (qtts/quant/fp8.py:52-89):
``fp8_weight`` is the column-major [K, N] view of a per-channel e4m3 weight,
``fp8_scale`` is [1, N] fp32, and ``apply`` quantizes the activations per token
(amax / 448, clamped at 1e-6) before the scaled GEMM. Both steps run on the
sm_100a library: one activation-quantization kernel and one fp8 GEMM whose
epilogue applies the row scale, the column scale and the bias.

:class:`Fp8WeightOnlyMethod` is the variant the reference leaves unimplemented
(fp8.py:92-122) because its only available form dequantizes into global
memory. Here it runs on the same fused weight-streaming design as int8
weight-only; until that kernel lands it raises like the reference.
"""

from __future__ import annotations

import torch

from ..layers.linear import LinearBase
from ..utils import get_logger
from .base import QuantMethodBase
from .kernels import fp8_quant_rows, fp8_scaled_mm, kernel_available, quantize_fp8_rows

logger = get_logger("quant.fp8")

#: Largest finite magnitude in e4m3.
_FP8_MAX = 448.0


def quantize_weight_fp8(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel e4m3. Returns ``(fp8 weight, fp32 scale)``.

    Same arithmetic as fp8.py:45-49 (amax / 448 clamped at 1e-12, round to
    nearest even), computed by the library on the GPU.
    """
    return quantize_fp8_rows(weight)


class Fp8Method(QuantMethodBase):
    """W8A8 e4m3: per-token activation scales, per-channel weight scales."""

    name = "fp8"

    def __init__(self) -> None:
        available, reason = kernel_available()
        if not available:
            raise RuntimeError(f"fp8 needs the sm_100a kernels of qtts_b200: {reason}")

    def process_weights(self, layer: LinearBase) -> None:
        q, scale = quantize_weight_fp8(layer.weight)
        # Same buffer layout as the reference: the [N, K] row-major weight kept
        # as its column-major [K, N] transpose view.
        layer.register_buffer("fp8_weight", q.t(), persistent=False)
        layer.register_buffer("fp8_scale", scale.reshape(1, -1), persistent=False)
        layer.weight = torch.nn.Parameter(
            torch.empty(0, dtype=layer.weight.dtype, device=layer.weight.device), requires_grad=False
        )

    def applies_to(self, layer: LinearBase) -> bool:
        return getattr(layer, "fp8_weight", None) is not None

    def apply(self, layer: LinearBase, x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        shape = x.shape
        xq, scale_x = fp8_quant_rows(x)
        out = fp8_scaled_mm(
            xq,
            scale_x,
            layer.fp8_weight.t(),  # type: ignore[attr-defined]
            layer.fp8_scale,  # type: ignore[attr-defined]
            bias,
            x.dtype,
        )
        return out.reshape(*shape[:-1], layer.out_features)


class Fp8WeightOnlyMethod(QuantMethodBase):
    """fp8 weights, bf16 activations -- not implemented yet, as in the reference."""

    name = "fp8_weight_only"

    def __init__(self, calibrate: bool = True, calibration_batch: int = 16) -> None:
        raise NotImplementedError(
            "fp8 weight-only is not implemented: use --quant-method int8_weight_only for the same "
            "footprint, or --quant-method fp8 for the W8A8 path."
        )
