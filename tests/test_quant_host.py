"""Host-side logic of the drop-in quantization API, on CPU.

Mirrors what the reference's API does without touching a GPU: QuantConfig and
its flags (qtts/config.py:50-98, 387-432), the exclude/convert/decline walk and
byte report of quantize_module (qtts/quant/base.py:74-113, checked against the
report the reference itself produced), method selection (base.py:116-130),
calibration's decline-on-failure (calibrate.py:97-103), and the LinearBase
hook (linear.py:57-60). The GPU kernels are replaced by a fake method here, the
way the reference's scheduler tests use a fake runner.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from qtts_b200.config import QuantConfig, add_quant_args, quant_config_from_args
from qtts_b200.layers.linear import LinearBase, MergedLinear, iter_linears
from qtts_b200.quant import apply_quantization, build_method, calibrate, quantize_module
from qtts_b200.quant import kernels as qk
from qtts_b200.quant.base import QuantMethodBase

GOLDEN = Path(__file__).resolve().parent / "golden"


# ---------------------------------------------------------------- config


def test_quant_config_defaults():
    cfg = QuantConfig()
    assert not cfg.enabled
    assert cfg.targets == ("talker",)
    assert cfg.excludes("layers.0.codec_head") and cfg.excludes("lm_head.3")
    assert not cfg.excludes("layers.3.mlp.down_proj")
    cfg = QuantConfig(method="int8_weight_only")
    assert cfg.enabled and cfg.weight_only and cfg.targets_submodel("talker")
    assert not cfg.targets_submodel("code2wav")


def _parse(argv):
    p = add_quant_args(argparse.ArgumentParser())
    return quant_config_from_args(p.parse_args(argv))


def test_flags_round_trip():
    cfg = _parse(["--quantization", "int8_weight_only"])
    assert cfg.method == "int8_weight_only" and cfg.calibrate is True
    cfg = _parse(["--quant-method", "int8_weight_only", "--no-quant-calibrate"])
    assert cfg.calibrate is False
    cfg = _parse(["--quant-method", "fp8", "--quant-calibrate", "--quant-targets", "talker,code2wav"])
    assert cfg.method == "fp8" and cfg.calibrate is True and cfg.targets == ("talker", "code2wav")
    # "" splits into no parts: every linear is eligible
    cfg = _parse(["--quantization", "int8_weight_only", "--quant-exclude-substrings", ""])
    assert cfg.exclude_substrings == ()
    assert _parse([]) == QuantConfig()


# ---------------------------------------------------------------- LinearBase


class _Recorder:
    name = "recorder"

    def __init__(self):
        self.calls = 0

    def process_weights(self, layer):
        pass

    def apply(self, layer, x, bias):
        self.calls += 1
        return torch.zeros(*x.shape[:-1], layer.out_features)


def test_linear_hook():
    lin = LinearBase(8, 4, bias=True, dtype=torch.float32)
    lin.weight.data.normal_()
    lin.bias.data.normal_()
    x = torch.randn(3, 8)
    torch.testing.assert_close(lin(x), F.linear(x, lin.weight, lin.bias))
    rec = _Recorder()
    lin.quant_method = rec
    assert lin(x).shape == (3, 4) and rec.calls == 1
    assert "quant=recorder" in lin.extra_repr()


def test_merged_linear_partitions():
    m = MergedLinear(8, [4, 2, 2], dtype=torch.float32)
    assert m.out_features == 8 and m.offsets == [0, 4, 6, 8]
    m.load_partition(1, torch.ones(2, 8))
    assert m.weight.data[4:6].eq(1).all()
    with pytest.raises(ValueError):
        m.load_partition(0, torch.ones(3, 8))
    with pytest.raises(ValueError):
        m.load_bias_partition(0, torch.ones(4))
    parts = m.split(torch.arange(8.0).reshape(1, 8))
    assert [p.shape[-1] for p in parts] == [4, 2, 2]


# ---------------------------------------------------------------- quantize_module report


class FakeInt8WeightOnly(QuantMethodBase):
    """Same buffers as Int8WeightOnlyMethod, computed by the CPU oracle."""

    name = "int8_weight_only"

    def __init__(self, decline=()):
        self.decline = set(decline)

    def process_weights(self, layer):
        if id(layer) in self.decline:
            layer.register_buffer("int8_weight", None, persistent=False)
            return
        q, s = oracle.quantize_weight_per_channel(layer.weight.detach().float().numpy())
        layer.register_buffer("int8_weight", torch.from_numpy(q), persistent=False)
        layer.register_buffer("int8_scale", torch.from_numpy(s).to(layer.weight.dtype), persistent=False)
        layer.weight = torch.nn.Parameter(torch.empty(0, dtype=layer.weight.dtype), requires_grad=False)

    def applies_to(self, layer):
        return getattr(layer, "int8_weight", None) is not None


def _reference_tree():
    # The module tree used by tests/golden/make_golden.py (reference layer names).
    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.qkv_proj = MergedLinear(64, [64, 32, 32], dtype=torch.bfloat16)
            self.o_proj = LinearBase(64, 64, dtype=torch.bfloat16)

    class Mlp(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_up_proj = MergedLinear(64, [96, 96], dtype=torch.bfloat16)
            self.down_proj = LinearBase(96, 64, bias=True, dtype=torch.bfloat16)

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = Attn()
            self.mlp = Mlp()

    class Talker(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = torch.nn.ModuleList([Block(), Block()])
            self.codec_head = LinearBase(64, 80, dtype=torch.bfloat16)
            self.text_projection = LinearBase(64, 64, dtype=torch.bfloat16)

    class Predictor(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = torch.nn.ModuleList([Block()])
            self.lm_head = torch.nn.ModuleList([LinearBase(64, 48, dtype=torch.bfloat16) for _ in range(3)])
            self.small_to_mtp_projection = LinearBase(64, 64, bias=True, dtype=torch.bfloat16)

    talker, predictor = Talker(), Predictor()
    for mod in (talker, predictor):
        for p in mod.parameters():
            p.data.normal_(0.0, 0.02)
    return talker, predictor


@pytest.mark.parametrize("label,excl", [("default", None), ("all", ())])
def test_quantize_module_report_matches_reference(label, excl):
    expected = json.loads((GOLDEN / "quantize_report.json").read_text())[label]
    talker, predictor = _reference_tree()
    kwargs = {"method": "int8_weight_only", "calibrate": False}
    if excl is not None:
        kwargs["exclude_substrings"] = excl
    cfg = QuantConfig(**kwargs)
    method = FakeInt8WeightOnly()
    got = {
        "talker": quantize_module(talker, method, cfg, "talker"),
        "code_predictor": quantize_module(predictor, method, cfg, "code_predictor"),
    }
    assert got == expected
    for name, layer in iter_linears(talker):
        if cfg.excludes(name):
            assert layer.quant_method is None
        else:
            assert layer.quant_method is method and layer.int8_weight.dtype == torch.int8
            assert layer.int8_scale.dtype == torch.bfloat16 and layer.weight.numel() == 0


def test_declined_layer_keeps_f_linear():
    talker, _ = _reference_tree()
    layers = [l for _, l in iter_linears(talker)]
    method = FakeInt8WeightOnly(decline={id(layers[0])})
    rep = quantize_module(talker, method, QuantConfig(method="int8_weight_only", exclude_substrings=()), "t")
    assert rep["declined"] == 1 and rep["converted"] == len(layers) - 1
    assert layers[0].quant_method is None and layers[0].weight.numel() > 0


def test_apply_quantization_routing(monkeypatch):
    import qtts_b200.quant.base as base

    monkeypatch.setattr(base, "build_method", lambda cfg, calibration_batch=16: FakeInt8WeightOnly())
    talker, predictor = _reference_tree()
    assert apply_quantization(QuantConfig(), talker=talker) == {}
    rep = apply_quantization(QuantConfig(method="int8_weight_only"), talker=talker, code_predictor=predictor)
    assert set(rep) == {"talker", "code_predictor"}
    with pytest.raises(ValueError):
        apply_quantization(QuantConfig(method="int8_weight_only", targets=("vocoder",)), talker=talker)


def test_build_method_selection():
    with pytest.raises(ValueError):
        build_method(QuantConfig(method="int4"))  # type: ignore[arg-type]
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="sm_100a"):
            build_method(QuantConfig(method="int8"))
        with pytest.raises(RuntimeError, match="sm_100a"):
            build_method(QuantConfig(method="int8_weight_only"))
        with pytest.raises(RuntimeError, match="fp8 quantization unavailable"):
            build_method(QuantConfig(method="fp8"))


def test_int8_w8a8_method_needs_the_library():
    # Int8Method runs on the sm_100a kernels (no CPU or torch._int_mm fallback).
    from qtts_b200.quant.int8 import Int8Method

    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="sm_100a"):
            Int8Method()


# ---------------------------------------------------------------- calibration


def test_calibration_declines_on_failure():
    calibrate.clear_cache()

    def boom():
        raise RuntimeError("capture failed")

    key = ("int8_wo", 1, 1, 1, "x")
    assert calibrate.worth_quantizing(boom, boom, key=key) is False
    assert calibrate._CACHE[key] is False
    # cached: the callables are not called again
    assert calibrate.worth_quantizing(None, None, key=key) is False  # type: ignore[arg-type]


def test_choose_variant_skips_failures():
    calibrate.clear_cache()

    def boom():
        raise RuntimeError("not applicable")

    assert calibrate.choose_variant({0x101: boom, 0x102: boom}, key=("v",)) == 0
    assert calibrate.lookup_variant(("v",)) == 0
    calibrate.clear_cache()
    assert calibrate.lookup_variant(("v",)) is None


# ---------------------------------------------------------------- no CPU fallback


def test_kernels_refuse_cpu_tensors():
    x = torch.randn(2, 32, dtype=torch.bfloat16)
    q = torch.zeros(16, 32, dtype=torch.int8)
    s = torch.ones(16, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        qk.w8_gemm(x, q, s)
    with pytest.raises(RuntimeError):
        qk.quantize_int8_rows(torch.randn(4, 4))
