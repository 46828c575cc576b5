"""Quantization configuration and its command-line flags.

``QuantConfig`` keeps the fields, defaults and helpers of the reference
(qtts/config.py:50-98). ``add_quant_args`` / ``quant_config_from_args``
reproduce how the reference turns the dataclass into flags
(config.py:366-414, 417-432): ``--quant-method`` (alias ``--quantization``),
``--quant-targets`` and ``--quant-exclude-substrings`` as comma-separated
tuples (an empty string gives ``()``), and ``--quant-calibrate`` /
``--no-quant-calibrate``.
"""

from __future__ import annotations

import argparse
import dataclasses
from dataclasses import dataclass
from typing import Any, Literal

METHODS = ("none", "fp8", "fp8_weight_only", "int8", "int8_weight_only")


@dataclass
class QuantConfig:
    """Weight/activation quantization of the linear layers."""

    method: Literal["none", "fp8", "fp8_weight_only", "int8", "int8_weight_only"] = "none"
    #: Which submodels to quantize; Code2Wav is not in the default.
    targets: tuple[str, ...] = ("talker",)
    #: Layers whose name contains any of these keep full precision.
    exclude_substrings: tuple[str, ...] = (
        "lm_head",
        "codec_head",
        "text_projection",
        "small_to_mtp_projection",
    )
    #: Time each distinct linear shape both ways at load and only replace the
    #: GEMM where the quantized one measures faster.
    calibrate: bool = True

    @property
    def enabled(self) -> bool:
        return self.method != "none"

    @property
    def weight_only(self) -> bool:
        return self.method.endswith("_weight_only")

    def targets_submodel(self, name: str) -> bool:
        return self.enabled and name in self.targets

    def excludes(self, layer_name: str) -> bool:
        return any(s in layer_name for s in self.exclude_substrings)


def add_quant_args(parser: argparse.ArgumentParser) -> argparse.ArgumentParser:
    """Add the ``--quant-*`` flags and the ``--quantization`` alias."""
    for f in dataclasses.fields(QuantConfig):
        flag = f"--quant-{f.name.replace('_', '-')}"
        ann = f.type if isinstance(f.type, str) else getattr(f.type, "__name__", "str")
        if ann.startswith("tuple"):
            parser.add_argument(flag, type=str, default=None)
        elif ann.startswith("bool") or isinstance(f.default, bool):
            parser.add_argument(flag, action=argparse.BooleanOptionalAction, default=None)
        else:
            parser.add_argument(flag, type=str, default=None)
    parser.add_argument("--quantization", type=str, default=None, help="alias for --quant-method")
    return parser


def quant_config_from_args(args: argparse.Namespace) -> QuantConfig:
    """Build a QuantConfig from the flags that were actually passed."""
    kwargs: dict[str, Any] = {}
    for f in dataclasses.fields(QuantConfig):
        value = getattr(args, f"quant_{f.name}", None)
        if value is None:
            continue
        ann = f.type if isinstance(f.type, str) else getattr(f.type, "__name__", "str")
        if ann.startswith("tuple"):
            kwargs[f.name] = tuple(s.strip() for s in str(value).split(",") if s.strip())
        else:
            kwargs[f.name] = value
    if getattr(args, "quantization", None):
        kwargs["method"] = args.quantization
    return QuantConfig(**kwargs)
