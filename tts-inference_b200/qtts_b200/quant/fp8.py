"""fp8 (e4m3) quantization methods.

:class:`Fp8Method` keeps the reference's W8A8 contract (qtts/quant/fp8.py:52-89):
``fp8_weight`` is the column-major [K, N] view of a per-channel e4m3 weight,
``fp8_scale`` is [1, N] fp32, and ``apply`` quantizes the activations per token
(amax / 448, clamped at 1e-6) before the scaled GEMM. Both steps run on the
sm_100a library: one activation-quantization kernel and one fp8 GEMM whose
epilogue applies the row scale, the column scale and the bias.

:class:`Fp8WeightOnlyMethod` is the variant the reference leaves unimplemented
(fp8.py:92-122) because its only available form dequantizes into global
memory. Here it runs on the same fused weight-streaming kernels as int8
weight-only, with the e4m3 weights converted in registers.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ..layers.linear import LinearBase
from ..utils import get_logger
from .base import QuantMethodBase
from .calibrate import worth_quantizing
from .kernels import fp8_quant_rows, fp8_scaled_mm, fp8w_gemm, kernel_available, quantize_fp8_rows

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
    """fp8 (e4m3) weights, bf16 activations, converted inside the GEMM.

    The reference leaves this method unimplemented (fp8.py:92-122): its only
    route would dequantize the weight into global memory on every call. Here
    the weight streams as e4m3 bytes into the same kernels as int8
    weight-only and is converted to 16-bit floats in registers (one
    conversion per two weights, exact), with the per-channel scale applied
    after the fp32 K loop. Buffers follow :class:`Fp8Method`: ``fp8_weight``
    is the [K, N] transposed view of the [N, K] e4m3 weight, ``fp8_scale``
    [1, N] fp32 (amax / 448, fp8.py:45-49). With ``calibrate`` a layer keeps
    F.linear where the quantized GEMM measures slower at
    ``calibration_batch`` rows, as int8 weight-only does.
    """

    name = "fp8_weight_only"

    def __init__(self, calibrate: bool = True, calibration_batch: int = 16) -> None:
        available, reason = kernel_available()
        if not available:
            raise RuntimeError(f"fp8 weight-only needs the sm_100a kernels of qtts_b200: {reason}")
        self.calibrate = calibrate
        self.calibration_batch = calibration_batch
        self.quantized = 0
        self.declined = 0

    def _profitable(self, layer: LinearBase, q: torch.Tensor, scale: torch.Tensor) -> bool:
        if not self.calibrate:
            return True
        weight = layer.weight
        if weight.device.type != "cuda":
            return False
        rows = max(1, self.calibration_batch)
        x = torch.zeros(rows, layer.in_features, device=weight.device, dtype=weight.dtype)
        return worth_quantizing(
            lambda: fp8w_gemm(x, q, scale, None),
            lambda: F.linear(x, weight, None),
            key=("fp8_wo", layer.out_features, layer.in_features, rows, str(weight.dtype)),
        )

    def process_weights(self, layer: LinearBase) -> None:
        q, scale = quantize_weight_fp8(layer.weight)
        if not self._profitable(layer, q, scale):
            self.declined += 1
            layer.register_buffer("fp8_weight", None, persistent=False)
            return
        layer.register_buffer("fp8_weight", q.t(), persistent=False)
        layer.register_buffer("fp8_scale", scale.reshape(1, -1), persistent=False)
        layer.weight = torch.nn.Parameter(
            torch.empty(0, dtype=layer.weight.dtype, device=layer.weight.device), requires_grad=False
        )
        self.quantized += 1

    def applies_to(self, layer: LinearBase) -> bool:
        return getattr(layer, "fp8_weight", None) is not None

    def apply(self, layer: LinearBase, x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        return fp8w_gemm(
            x,
            layer.fp8_weight.t(),  # type: ignore[attr-defined]
            layer.fp8_scale.reshape(-1),  # type: ignore[attr-defined]
            bias,
        )
