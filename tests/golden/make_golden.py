"""Generate the golden vectors that pin the CPU oracle to the reference.

Run from the repository root with the reference checkout on the path:

    QTTS_REFERENCE_DIR=<path to danielhua23/tts-inference> python tests/golden/make_golden.py

It imports the reference's own ``qtts`` package (and its tuning script) and
records, on seeded CPU inputs:

* ``quantize_weight_per_channel`` (qtts/quant/int8.py:45-56) on fp32 and bf16
  weights, including an all-zero row (the 1e-12 floor);
* ``quantize_weight_fp8`` (qtts/quant/fp8.py:45-49);
* the per-token activation quantization of ``Fp8Method.apply``
  (qtts/quant/fp8.py:72-89), captured by replacing ``torch._scaled_mm`` with a
  recorder (the real one needs a GPU) for bf16, fp16 and fp32 activations,
  including an all-zero row and a row below the 1e-6 floor;
* the tuning script's ``quantize`` and ``naive_dequant_linear``
  (examples/kernels/tune_w8_gemm.py:73-85) -- the eager dequantize-then-matmul
  the kernels are checked against;
* ``Int8Method`` (qtts/quant/int8.py:120-155) on bf16, fp16 and fp32 layers
  with a bias: the int8 weight and scale, the activation codes (captured from
  ``torch._int_mm``, which runs on the CPU) and the output, including an
  all-zero row, a row below the 1e-6 floor and a large row;
* the byte/convert report of ``apply_quantization`` / ``quantize_module``
  (qtts/quant/base.py:74-113, 155-183) with int8 weight-only, calibration
  off, on a small module tree with the reference's layer names;
* ``RMSNorm`` (qtts/layers/norm.py:123-137, the eager form the CPU runs) on
  bf16, fp16 and fp32 rows of the model's widths, including an all-zero row
  and a tiny one (the eps floor);
* the SwiGLU product ``F.silu(gate) * up`` of ``GatedMLP.forward``
  (qtts/layers/activation.py:147) on bf16 and fp16 ``[gate | up]`` rows split
  with ``MergedLinear.split`` (qtts/layers/linear.py:99-100).

The reference is not needed afterwards: tests read only the files written
here (``quant_golden.npz``, ``quantize_report.json``).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("QTTS_REFERENCE_DIR", "/root/reference"))
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REF / "examples" / "kernels"))

import qtts.layers.norm as ref_norm  # noqa: E402
import qtts.quant.fp8 as ref_fp8  # noqa: E402
import qtts.quant.int8 as ref_int8  # noqa: E402
import tune_w8_gemm as ref_tune  # noqa: E402
from qtts.config import QuantConfig  # noqa: E402
from qtts.layers.linear import LinearBase, MergedLinear  # noqa: E402
from qtts.quant import apply_quantization  # noqa: E402


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().numpy()


def main() -> None:
    g = torch.Generator().manual_seed(0)
    out: dict[str, np.ndarray] = {}

    # -- weights: 48 x 160, rows of different magnitude, one all-zero row --
    n, k = 48, 160
    w = torch.randn(n, k, generator=g) * 0.02
    w[5] *= 40.0
    w[7] = 0.0
    w[11, :] = torch.linspace(-1.0, 1.0, k)
    out["w_f32"] = f32(w)
    q, s = ref_int8.quantize_weight_per_channel(w)
    out["int8_q_f32"] = q.numpy()
    out["int8_scale_f32"] = s.numpy()
    wb = w.to(torch.bfloat16)
    out["w_bf16"] = f32(wb)
    q, s = ref_int8.quantize_weight_per_channel(wb)
    out["int8_q_bf16"] = q.numpy()
    out["int8_scale_bf16"] = s.numpy()

    qf, sf = ref_fp8.quantize_weight_fp8(w)
    out["fp8_q_f32"] = qf.view(torch.uint8).numpy()
    out["fp8_scale_f32"] = sf.numpy()
    qf, sf = ref_fp8.quantize_weight_fp8(wb)
    out["fp8_q_bf16"] = qf.view(torch.uint8).numpy()
    out["fp8_scale_bf16"] = sf.numpy()

    # -- fp8 activation quantization, captured from Fp8Method.apply --
    captured: dict[str, torch.Tensor] = {}

    def recorder(a, b, scale_a=None, scale_b=None, bias=None, out_dtype=None, **_):
        captured["q"] = a
        captured["scale"] = scale_a
        return torch.zeros(a.shape[0], b.shape[1], dtype=out_dtype)

    method = ref_fp8.Fp8Method()
    layer = LinearBase(k, n, bias=False, dtype=torch.float32)
    layer.weight.data.copy_(w)
    method.process_weights(layer)
    real = torch._scaled_mm
    torch._scaled_mm = recorder
    try:
        for name, dtype in (("bf16", torch.bfloat16), ("fp16", torch.float16), ("f32", torch.float32)):
            x = torch.randn(6, k, generator=g)
            x[1] = 0.0
            x[2] = x[2] * 1e-8  # amax below the 1e-6 floor
            x[3] = x[3] * 300.0
            x = x.to(dtype)
            method.apply(layer, x, None)
            out[f"act_x_{name}"] = f32(x)
            out[f"act_q_{name}"] = captured["q"].view(torch.uint8).numpy()
            out[f"act_scale_{name}"] = captured["scale"].reshape(-1).numpy()
    finally:
        torch._scaled_mm = real

    # -- tuning script: quantize + naive eager dequant linear (bf16) --
    wt = (torch.randn(n, k, generator=g) / (k**0.5)).to(torch.bfloat16)
    packed, scale = ref_tune.quantize(wt)
    out["tune_w"] = f32(wt)
    out["tune_q"] = packed.numpy()
    out["tune_scale"] = f32(scale)
    for m in (1, 3, 8):
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        y = ref_tune.naive_dequant_linear(x, packed, scale, torch.bfloat16)
        out[f"naive_x_m{m}"] = f32(x)
        out[f"naive_y_m{m}"] = f32(y)

    # -- Int8Method (W8A8): activation codes captured from torch._int_mm, and the output --
    gi = torch.Generator().manual_seed(7)
    wi = torch.randn(n, k, generator=gi) * 0.02
    bi = torch.randn(n, generator=gi)
    out["w8a8_w"] = f32(wi)
    out["w8a8_bias"] = f32(bi)
    seen: dict[str, torch.Tensor] = {}
    real_int_mm = torch._int_mm

    def int_mm_recorder(a, b):
        seen["q"] = a
        return real_int_mm(a, b)

    torch._int_mm = int_mm_recorder
    try:
        for name, dtype in (("bf16", torch.bfloat16), ("fp16", torch.float16), ("f32", torch.float32)):
            method = ref_int8.Int8Method()
            layer = LinearBase(k, n, bias=True, dtype=dtype)
            layer.weight.data.copy_(wi.to(dtype))
            layer.bias.data.copy_(bi.to(dtype))
            method.process_weights(layer)
            out[f"w8a8_wq_{name}"] = layer.int8_weight.t().contiguous().numpy()
            out[f"w8a8_ws_{name}"] = layer.int8_scale.numpy()
            x = torch.randn(6, k, generator=gi)
            x[1] = 0.0
            x[2] = x[2] * 1e-8  # amax below the 1e-6 floor
            x[3] = x[3] * 300.0
            x = x.to(dtype)
            y = method.apply(layer, x, layer.bias)
            out[f"w8a8_x_{name}"] = f32(x)
            out[f"w8a8_q_{name}"] = seen["q"][: x.shape[0]].numpy()  # apply pads to 17 rows
            out[f"w8a8_y_{name}"] = f32(y)
    finally:
        torch._int_mm = real_int_mm

    # -- RMSNorm (eager form) and SiLU·up --
    gn = torch.Generator().manual_seed(11)
    for name, dtype in (("bf16", torch.bfloat16), ("fp16", torch.float16), ("f32", torch.float32)):
        for width in (128, 1024, 2048):
            norm = ref_norm.RMSNorm(width, eps=1e-6, dtype=dtype, backend="eager")
            norm.weight.data.copy_((1.0 + 0.1 * torch.randn(width, generator=gn)).to(dtype))
            x = torch.randn(6, width, generator=gn) * 3.0
            x[1] = 0.0
            x[2] = x[2] * 1e-5
            x[4] = x[4] * 200.0
            x = x.to(dtype)
            with torch.no_grad():
                y = norm(x)
            out[f"rms_x_{name}_{width}"] = f32(x)
            out[f"rms_w_{name}_{width}"] = f32(norm.weight)
            out[f"rms_y_{name}_{width}"] = f32(y)
    merged = MergedLinear(8, [384, 384], bias=False, dtype=torch.float32)
    for name, dtype in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
        gate_up = (torch.randn(5, 768, generator=gn) * 4.0).to(dtype)
        gate_up[0, :8] = torch.tensor([0.0, -0.0, 20.0, -20.0, 90.0, -90.0, 1e-3, -1e-3]).to(dtype)
        gate, up = merged.split(gate_up)
        y = torch.nn.functional.silu(gate) * up
        out[f"silu_gate_up_{name}"] = f32(gate_up)
        out[f"silu_y_{name}"] = f32(y)

    np.savez_compressed(HERE / "quant_golden.npz", **out)

    # -- quantize_module byte report on the reference layer names --
    torch.manual_seed(0)

    class Attn(torch.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.qkv_proj = MergedLinear(64, [64, 32, 32], dtype=torch.bfloat16)
            self.o_proj = LinearBase(64, 64, dtype=torch.bfloat16)

    class Mlp(torch.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.gate_up_proj = MergedLinear(64, [96, 96], dtype=torch.bfloat16)
            self.down_proj = LinearBase(96, 64, bias=True, dtype=torch.bfloat16)

    class Block(torch.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.self_attn = Attn()
            self.mlp = Mlp()

    class Talker(torch.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.layers = torch.nn.ModuleList([Block(), Block()])
            self.codec_head = LinearBase(64, 80, dtype=torch.bfloat16)
            self.text_projection = LinearBase(64, 64, dtype=torch.bfloat16)

    class Predictor(torch.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.layers = torch.nn.ModuleList([Block()])
            self.lm_head = torch.nn.ModuleList([LinearBase(64, 48, dtype=torch.bfloat16) for _ in range(3)])
            self.small_to_mtp_projection = LinearBase(64, 64, bias=True, dtype=torch.bfloat16)

    reports = {}
    for label, excl in (("default", None), ("all", ())):
        talker, predictor = Talker(), Predictor()
        for mod in (talker, predictor):
            for p in mod.parameters():
                p.data.normal_(0.0, 0.02)
        kwargs = {"method": "int8_weight_only", "calibrate": False}
        if excl is not None:
            kwargs["exclude_substrings"] = excl
        cfg = QuantConfig(**kwargs)
        reports[label] = apply_quantization(cfg, talker=talker, code_predictor=predictor, calibration_batch=8)
    with open(HERE / "quantize_report.json", "w") as fh:
        json.dump(reports, fh, indent=1, sort_keys=True)
    print(f"wrote {HERE / 'quant_golden.npz'} and {HERE / 'quantize_report.json'}")


if __name__ == "__main__":
    main()
