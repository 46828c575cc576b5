"""Quantization dispatch: pick a method, attach it to the chosen linears.

Same contract as qtts/quant/base.py. A quant method is an object assigned to
``LinearBase.quant_method`` after the checkpoint is loaded
(base.py:1-27); ``quantize_module`` walks the linears, skips excluded names,
lets the method convert or decline each layer and reports bytes before and
after (base.py:74-113); ``build_method`` maps the method name to a class
(base.py:116-130); ``apply_quantization`` quantizes the submodels named in
``QuantConfig.targets``, the code predictor following the talker target
(base.py:155-183).

What changes is underneath: the methods call the sm_100a kernels of this
package, and ``fp8_supported`` asks for this library and a compute-capability
10.x GPU instead of ``torch._scaled_mm``.
"""

from __future__ import annotations

import torch
from torch import nn

from ..config import QuantConfig
from ..layers.linear import LinearBase, iter_linears
from ..utils import get_logger, human_bytes

logger = get_logger("quant")


class QuantMethodBase:
    """Base for the assign-after-load quant methods (base.py:41-63)."""

    name = "base"

    def process_weights(self, layer: LinearBase) -> None:
        raise NotImplementedError

    def applies_to(self, layer: LinearBase) -> bool:
        """Whether ``process_weights`` actually converted this layer.

        A method may decline a layer (calibration found it slower than the
        unquantized GEMM); declining leaves ``quant_method`` unset so the layer
        keeps ``F.linear``.
        """
        return True

    def apply(self, layer: LinearBase, x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        raise NotImplementedError


def _param_bytes(module: nn.Module) -> int:
    return sum(p.numel() * p.element_size() for p in module.parameters(recurse=True))


def _buffer_bytes(module: nn.Module) -> int:
    return sum(b.numel() * b.element_size() for b in module.buffers(recurse=True))


def quantize_module(module: nn.Module, method: QuantMethodBase, config: QuantConfig, label: str) -> dict[str, int]:
    """Attach ``method`` to every eligible :class:`LinearBase` under ``module``.

    Returns the byte counts before and after and how many layers were
    converted, excluded by name and declined (base.py:74-113).
    """
    before = _param_bytes(module) + _buffer_bytes(module)
    converted = 0
    excluded = 0
    declined = 0
    for name, layer in iter_linears(module):
        if config.excludes(name):
            excluded += 1
            continue
        method.process_weights(layer)
        if not method.applies_to(layer):
            declined += 1
            continue
        layer.quant_method = method
        converted += 1
    after = _param_bytes(module) + _buffer_bytes(module)
    logger.info(
        "%s: %s on %d linears (%d excluded by name, %d declined as not faster), %s -> %s",
        label,
        method.name,
        converted,
        excluded,
        declined,
        human_bytes(before),
        human_bytes(after),
    )
    return {
        "converted": converted,
        "excluded": excluded,
        "declined": declined,
        "bytes_before": before,
        "bytes_after": after,
    }


def build_method(config: QuantConfig, calibration_batch: int = 16) -> QuantMethodBase:
    from .fp8 import Fp8Method, Fp8WeightOnlyMethod
    from .int8 import Int8Method, Int8WeightOnlyMethod

    method = config.method
    if method in ("fp8", "fp8_weight_only"):
        supported, reason = fp8_supported()
        if not supported:
            raise RuntimeError(f"fp8 quantization unavailable: {reason}")
        if method.endswith("_weight_only"):
            return Fp8WeightOnlyMethod(calibrate=config.calibrate, calibration_batch=calibration_batch)
        return Fp8Method()
    if method == "int8_weight_only":
        return Int8WeightOnlyMethod(calibrate=config.calibrate, calibration_batch=calibration_batch)
    if method == "int8":
        return Int8Method()
    raise ValueError(f"unknown quantization method {method!r}")


def fp8_supported() -> tuple[bool, str]:
    """Whether the fp8 kernels can run here, and why not if they cannot.

    Checked up front, before any weight is touched (base.py:133-152).
    """
    if not torch.cuda.is_available():
        return False, "no CUDA device"
    if not hasattr(torch, "float8_e4m3fn"):
        return False, f"torch {torch.__version__} has no float8_e4m3fn dtype"
    from .kernels import kernel_available

    ok, reason = kernel_available()
    if not ok:
        return False, reason
    return True, ""


def apply_quantization(
    config: QuantConfig,
    *,
    talker: nn.Module | None = None,
    code_predictor: nn.Module | None = None,
    code2wav: nn.Module | None = None,
    calibration_batch: int = 16,
) -> dict[str, dict[str, int]]:
    """Quantize the submodels named in ``config.targets``. Call after loading."""
    if not config.enabled:
        return {}
    unknown = set(config.targets) - {"talker", "code_predictor", "code2wav"}
    if unknown:
        raise ValueError(f"unknown quant targets {sorted(unknown)}; pick from talker, code_predictor, code2wav")
    method = build_method(config, calibration_batch=calibration_batch)
    report: dict[str, dict[str, int]] = {}
    if config.targets_submodel("talker"):
        if talker is not None:
            report["talker"] = quantize_module(talker, method, config, "talker")
        if code_predictor is not None:
            report["code_predictor"] = quantize_module(code_predictor, method, config, "code_predictor")
    if config.targets_submodel("code2wav") and code2wav is not None:
        report["code2wav"] = quantize_module(code2wav, method, config, "code2wav")
    return report
