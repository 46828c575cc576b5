"""Load-time calibration of ``Int8WeightOnlyMethod`` on the GPU.

The reference times its fused kernel against ``F.linear`` per layer shape at
``calibration_batch`` rows and keeps a layer on ``F.linear`` unless the kernel
wins by 5 % (qtts/quant/int8.py:79-93, qtts/quant/calibrate.py:77-114); a
failure inside the timing declines the layer (calibrate.py:97-103). The library
keeps that rule and also picks, per batch-row bucket, the fastest of its kernel
variants. Checked here on the four talker shapes with ``calibration_batch=8``:

* every quantized layer's output, through the variant calibration chose for
  each bucket, matches the oracle (max error 1e-2 of max|ref| and every output
  within one bf16 rounding of the exact value);
* a declined layer keeps its full-precision weight and its output is
  ``F.linear``'s, bit for bit;
* an exception raised inside the timed call declines the layer.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from conftest import require_b200
from qtts_b200 import _native as nat
from qtts_b200.layers.linear import LinearBase
from qtts_b200.quant import calibrate
from qtts_b200.quant import int8 as int8_mod
from qtts_b200.quant.int8 import Int8WeightOnlyMethod

pytestmark = pytest.mark.gpu

SHAPES = [("qkv", 4096, 2048), ("o_proj", 2048, 2048), ("gate_up", 12288, 2048), ("down_proj", 2048, 6144)]
BUCKET_ROWS = (1, 2, 4, 8)


@pytest.fixture(autouse=True)
def _device():
    require_b200()
    calibrate.clear_cache()
    nat.device_status(reset=True)
    yield
    calibrate.clear_cache()
    torch.cuda.synchronize()
    assert nat.device_status() == 0


def _layer(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    layer = LinearBase(k, n, dtype=torch.bfloat16, device="cuda")
    layer.weight.data.copy_((torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16))
    return layer


def _check(out, ref, what):
    out = out.float().cpu().numpy().astype(np.float64)
    err = oracle.rel_err(out, ref)
    assert err <= 1e-2, f"{what}: rel err {err:.3e}"
    bound = np.abs(ref) * 2.0**-8 + 1e-3 * np.abs(ref).max() + 1e-30
    assert not (np.abs(out - ref) > bound).any(), f"{what}: beyond one bf16 rounding"


@pytest.mark.parametrize("label,n,k", SHAPES)
def test_calibrated_layer_outputs(label, n, k):
    layer = _layer(n, k, seed=400)
    weight = layer.weight.detach().clone()
    method = Int8WeightOnlyMethod(calibrate=True, calibration_batch=8)
    method.process_weights(layer)
    g = torch.Generator().manual_seed(401)
    x = torch.randn(max(BUCKET_ROWS), k, generator=g).to(torch.bfloat16).cuda()
    if method.applies_to(layer):
        layer.quant_method = method
        q = layer.int8_weight.cpu().numpy()
        s = layer.int8_scale.float().cpu().numpy()
        ref = oracle.w8a16_reference(x.float().cpu().numpy(), q, s)
        chosen = {}
        for m in BUCKET_ROWS:
            chosen[m] = method.variant_for(n, k, m, torch.bfloat16)
            _check(layer(x[:m]), ref[:m], f"{label} M={m} variant {chosen[m]:#x}")
        assert layer.weight.numel() == 0
        print(f"\n{label}: quantized; variants per bucket {({m: hex(v) for m, v in chosen.items()})}")
    else:
        assert method.declined == 1
        assert layer.int8_weight is None and layer.quant_method is None
        assert torch.equal(layer.weight, weight)
        for m in BUCKET_ROWS:
            assert torch.equal(layer(x[:m]), F.linear(x[:m], weight))
        print(f"\n{label}: declined (F.linear faster by calibration)")


def test_exception_in_timed_call_declines(monkeypatch):
    n, k = 2048, 2048
    layer = _layer(n, k, seed=402)
    weight = layer.weight.detach().clone()

    def broken(*args, **kwargs):
        raise RuntimeError("simulated kernel failure during calibration")

    monkeypatch.setattr(int8_mod, "w8_gemm", broken)
    method = Int8WeightOnlyMethod(calibrate=True, calibration_batch=8)
    method.process_weights(layer)
    assert method.declined == 1 and method.quantized == 0
    assert not method.applies_to(layer)
    assert torch.equal(layer.weight, weight)
    x = torch.randn(8, k, generator=torch.Generator().manual_seed(403)).to(torch.bfloat16).cuda()
    assert torch.equal(layer(x), F.linear(x, weight))
