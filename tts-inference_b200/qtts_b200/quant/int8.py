"""int8 quantization methods.

:class:`Int8WeightOnlyMethod` keeps the reference's contract
(qtts/quant/int8.py:59-117): per-output-channel symmetric int8 weights stored
as ``int8_weight`` [N, K] and ``int8_scale`` [N] in the weight dtype,
calibration per distinct shape (``_profitable``), the full-precision weight
dropped after conversion, and ``apply`` computing
``x @ (int8_weight * int8_scale).T + bias``. The GEMM is the sm_100a kernel of
this package; calibration additionally records which kernel variant is fastest
for the shape, per batch-row bucket, and ``apply`` passes it along.

:class:`Int8Method` (W8A8, int8.py:120-155) keeps the reference's contract and
numbers on the same library: a per-token int8 activation quantizer and a
tcgen05 kind::i8 GEMM with the reference's epilogue arithmetic replace the
torch op sequence and ``torch._int_mm``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import _native as nat
from ..layers.linear import LinearBase
from ..utils import get_logger
from .base import QuantMethodBase
from .calibrate import choose_variant, lookup_variant, worth_quantizing
from .kernels import (
    i8_scaled_mm,
    int8_quant_rows,
    kernel_available,
    quantize_int8_rows,
    w8_gemm,
    w8_gemm_rmsnorm,
    w8_gemm_silu_mul,
)

logger = get_logger("quant.int8")

_INT8_MAX = 127.0
#: Batch-row buckets calibration times separately (the kernels' costs change
#: with the rows of an 8-wide MMA tile that are real, and between tiles).
_ROW_BUCKETS = (1, 2, 4, 8, 16, 32, 64)
#: Split-K factors and row tiles (groups of 16 weight rows per CTA) of the
#: split-K streaming kernel calibration chooses from.
_SPLITS = (1, 2, 4, 8)
_ROW_GROUPS = (1, 2, 4, 8)
#: Row tiles of the whole-K streaming kernel (16 * r rows per CTA).
_STREAM_ROWS = (1, 2, 3, 4, 6)
#: Split-K factors of the tcgen05 kernel (calibration candidates from the 16-row bucket up).
_UMMA_SPLITS = (1, 2, 4)


def variant_candidates(bucket: int) -> list[int]:
    """Kernel variants worth timing for up to ``bucket`` activation rows."""
    out = [nat.VARIANT_AUTO]
    if bucket <= 16:
        out += [nat.variant_skinny(s, r) for s in _SPLITS for r in _ROW_GROUPS]
        out += [nat.variant_stream(r) for r in _STREAM_ROWS]
    if bucket >= 16:
        out += [nat.variant_umma(s) for s in _UMMA_SPLITS]
    return out


def quantize_weight_per_channel(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel int8. Returns ``(int8 weight, fp32 scale)``.

    Same arithmetic as int8.py:45-56 -- fp32 absmax / 127 clamped at 1e-12,
    round half to even, clamp to +-127 -- computed on the GPU by the library
    (bit-exact with the reference's torch ops).
    """
    return quantize_int8_rows(weight)


def row_bucket(rows: int) -> int:
    for b in _ROW_BUCKETS:
        if rows <= b:
            return b
    return _ROW_BUCKETS[-1]


class Int8WeightOnlyMethod(QuantMethodBase):
    """int8 weights, bf16 activations, dequantized inside the GEMM."""

    name = "int8_weight_only"

    def __init__(self, calibrate: bool = True, calibration_batch: int = 16) -> None:
        available, reason = kernel_available()
        if not available:
            raise RuntimeError(f"int8 weight-only needs the sm_100a kernels of qtts_b200: {reason}")
        self.calibrate = calibrate
        self.calibration_batch = calibration_batch
        self.quantized = 0
        self.declined = 0

    # -- calibration ---------------------------------------------------------

    def _variant_key(self, n: int, k: int, bucket: int, dtype: torch.dtype) -> tuple:
        return ("int8_wo_variant", n, k, bucket, str(dtype))

    def _tune_variants(self, q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype) -> None:
        n, k = q.shape
        top = row_bucket(max(1, self.calibration_batch))
        for bucket in _ROW_BUCKETS:
            if bucket > top:
                break
            key = self._variant_key(n, k, bucket, dtype)
            if lookup_variant(key) is not None:
                continue
            x = torch.zeros(bucket, k, device=q.device, dtype=dtype)
            candidates = {
                v: (lambda v=v: w8_gemm(x, q, scale, None, variant=v)) for v in variant_candidates(bucket)
            }
            choose_variant(candidates, key=key)

    def _profitable(self, layer: LinearBase, q: torch.Tensor, scale: torch.Tensor) -> bool:
        if not self.calibrate:
            return True
        if not torch.cuda.is_available() or layer.weight.device.type != "cuda":
            return False
        weight = layer.weight
        rows = max(1, self.calibration_batch)
        self._tune_variants(q, scale, weight.dtype)
        x = torch.zeros(rows, layer.in_features, device=weight.device, dtype=weight.dtype)
        variant = self.variant_for(layer.out_features, layer.in_features, rows, weight.dtype)
        return worth_quantizing(
            lambda: w8_gemm(x, q, scale, None, variant=variant),
            lambda: F.linear(x, weight, None),
            key=("int8_wo", layer.out_features, layer.in_features, rows, str(weight.dtype)),
        )

    def variant_for(self, n: int, k: int, rows: int, dtype: torch.dtype) -> int:
        v = lookup_variant(self._variant_key(n, k, row_bucket(rows), dtype))
        return nat.VARIANT_AUTO if v is None else v

    # -- QuantMethodBase ------------------------------------------------------

    def process_weights(self, layer: LinearBase) -> None:
        q, scale = quantize_weight_per_channel(layer.weight)
        scale = scale.to(layer.weight.dtype)
        if not self._profitable(layer, q, scale):
            self.declined += 1
            # Leaving quant_method unset is what keeps the layer on F.linear.
            layer.register_buffer("int8_weight", None, persistent=False)
            return
        # Buffers rather than plain attributes so they follow module.to() and
        # are counted by the byte report of quantize_module.
        layer.register_buffer("int8_weight", q, persistent=False)
        layer.register_buffer("int8_scale", scale, persistent=False)
        # Drop the full-precision weight: keeping both would report a memory
        # saving that was not made.
        layer.weight = torch.nn.Parameter(
            torch.empty(0, dtype=layer.weight.dtype, device=layer.weight.device), requires_grad=False
        )
        self.quantized += 1

    def applies_to(self, layer: LinearBase) -> bool:
        return getattr(layer, "int8_weight", None) is not None

    def apply(self, layer: LinearBase, x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        rows = x.numel() // max(1, x.shape[-1])
        variant = self.variant_for(layer.out_features, layer.in_features, rows, x.dtype)
        return w8_gemm(x, layer.int8_weight, layer.int8_scale, bias, variant=variant)  # type: ignore[attr-defined]

    # -- fused activation prologues (LinearBase.forward_rmsnorm / forward_silu_mul) --

    def apply_rmsnorm(self, layer: LinearBase, x: torch.Tensor, norm_weight: torch.Tensor, eps: float,
                      bias: torch.Tensor | None) -> torch.Tensor:
        """``apply(layer, rms_norm(x), bias)`` with the norm inside the GEMM's activation staging."""
        rows = x.numel() // max(1, x.shape[-1])
        variant = self.variant_for(layer.out_features, layer.in_features, rows, x.dtype)
        return w8_gemm_rmsnorm(x, norm_weight, eps, layer.int8_weight, layer.int8_scale,  # type: ignore[attr-defined]
                               bias, variant=variant)

    def apply_silu_mul(self, layer: LinearBase, gate_up: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        """``apply(layer, silu(gate) * up, bias)`` of a ``[gate | up]`` input, fused the same way."""
        rows = gate_up.numel() // max(1, gate_up.shape[-1])
        variant = self.variant_for(layer.out_features, layer.in_features, rows, gate_up.dtype)
        return w8_gemm_silu_mul(gate_up, layer.int8_weight, layer.int8_scale, bias,  # type: ignore[attr-defined]
                                variant=variant)


class Int8Method(QuantMethodBase):
    """W8A8: per-token activation scales, per-channel weight scales, int8 GEMM.

    Same contract and numbers as the reference (qtts/quant/int8.py:120-155),
    on the sm_100a library instead of torch._int_mm: one kernel quantizes the
    activations per token (every step in the activation dtype, as torch does
    on a CUDA tensor) and one tcgen05 kind::i8 kernel computes the exact int32
    sums and the scaling ((acc * scale_x) * scale_w + bias, the reference's
    fp32 roundings). No 17-row padding. Buffers: ``int8_weight`` is the
    reference's [K, N] int8 layout as the transposed view of the K-major
    [N, K] array the kernel reads; ``int8_scale`` [N] fp32.
    """

    name = "int8"

    def __init__(self) -> None:
        available, reason = kernel_available()
        if not available:
            raise RuntimeError(f"int8 W8A8 needs the sm_100a kernels of qtts_b200: {reason}")

    def process_weights(self, layer: LinearBase) -> None:
        q, scale = quantize_weight_per_channel(layer.weight)
        layer.register_buffer("int8_weight", q.t(), persistent=False)
        layer.register_buffer("int8_scale", scale, persistent=False)
        layer.weight = torch.nn.Parameter(
            torch.empty(0, dtype=layer.weight.dtype, device=layer.weight.device), requires_grad=False
        )

    def applies_to(self, layer: LinearBase) -> bool:
        return getattr(layer, "int8_weight", None) is not None

    def apply(self, layer: LinearBase, x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        q, scale_x = int8_quant_rows(flat)
        out = i8_scaled_mm(
            q, scale_x, layer.int8_weight.t(), layer.int8_scale, bias, x.dtype  # type: ignore[attr-defined]
        )
        return out.reshape(*shape[:-1], layer.out_features)
