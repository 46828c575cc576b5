"""fp8 weight-only (e4m3 weights, 16-bit activations) through the C ABI, against the oracle.

The reference leaves Fp8WeightOnlyMethod unimplemented (qtts/quant/fp8.py:92-122);
the contract here is the W8A16 one with e4m3 weights: the exact decoded weight,
an fp32 K loop, the per-channel scale after it (float64 oracle:
``oracle.fp8_weight_only_reference``). Same bar as W8A16: within 1e-2 of max|ref|
and every output within one output rounding (+1e-3 max|ref|).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import require_b200
from qtts_b200 import _native as nat
from qtts_b200.layers.linear import LinearBase
from qtts_b200.quant import kernels as qk
from qtts_b200.quant.fp8 import Fp8WeightOnlyMethod

pytestmark = pytest.mark.gpu

SHAPES = [("qkv", 4096, 2048), ("o_proj", 2048, 2048), ("gate_up", 12288, 2048), ("down_proj", 2048, 6144)]


@pytest.fixture(scope="module", autouse=True)
def _device():
    require_b200()
    nat.device_status(reset=True)
    yield
    torch.cuda.synchronize()
    assert nat.device_status() == 0, "a kernel recorded a device-side failure"


def case(n, k, m, seed, x_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    x = torch.randn(m, k, generator=g).to(x_dtype)
    wq, ws = oracle.quantize_weight_fp8(w.numpy())
    dev = (x.cuda(), torch.from_numpy(wq).cuda().view(torch.float8_e4m3fn), torch.from_numpy(ws).cuda())
    return dev, (x.float().numpy(), wq, ws)


def check(out, ref, what, step=2.0**-8):
    out = out.float().cpu().numpy().astype(np.float64)
    err = oracle.rel_err(out, ref)
    assert err <= 1e-2, f"{what}: rel err {err:.3e}"
    bound = np.abs(ref) * step + 1e-3 * np.abs(ref).max() + 1e-30
    bad = np.abs(out - ref) > bound
    assert not bad.any(), f"{what}: {bad.sum()} elements beyond one output rounding (rel err {err:.3e})"


@pytest.mark.parametrize("label,n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 2, 8, 9, 16, 17, 32, 64])
def test_talker_shapes(label, n, k, m):
    (x, wq, ws), host = case(n, k, m, seed=90)
    out = qk.fp8w_gemm(x, wq, ws)
    check(out, oracle.fp8_weight_only_reference(*host), f"{label} M={m}")


VARIANTS = {
    "generic": nat.VARIANT_GENERIC,
    **{f"skinny{s}": nat.variant_skinny(s) for s in (1, 2, 4, 8)},
    **{f"umma{s}": nat.variant_umma(s) for s in (1, 2, 4)},
}


@pytest.mark.parametrize("variant", sorted(VARIANTS))
@pytest.mark.parametrize("m", [1, 16, 40])
def test_variants(variant, m):
    (x, wq, ws), host = case(2048, 6144, m, seed=91)
    if variant.startswith("skinny") and m > 16:
        # The split-K streaming kernel takes e4m3 weights up to 16 rows only.
        with pytest.raises(RuntimeError, match="inapplicable kernel variant"):
            qk.fp8w_gemm(x, wq, ws, variant=VARIANTS[variant])
        return
    out = qk.fp8w_gemm(x, wq, ws, variant=VARIANTS[variant])
    check(out, oracle.fp8_weight_only_reference(*host), f"{variant} M={m}")


def test_stream_variant_refused():
    (x, wq, ws), _ = case(256, 256, 4, seed=92)
    with pytest.raises(RuntimeError, match="inapplicable kernel variant"):
        qk.fp8w_gemm(x, wq, ws, variant=nat.variant_stream(0))


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_dtypes_and_bias(x_dtype):
    n, k, m = 1024, 2048, 5
    (x, wq, ws), host = case(n, k, m, seed=93, x_dtype=x_dtype)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(94)).to(x_dtype)
    ref = oracle.fp8_weight_only_reference(*host, bias=bias.float().numpy())
    out = qk.fp8w_gemm(x, wq, ws, bias.cuda())
    assert out.dtype == x_dtype
    step = {torch.bfloat16: 2.0**-8, torch.float16: 2.0**-11, torch.float32: 2.0**-22}[x_dtype]
    check(out, ref, f"{x_dtype}", step)


@pytest.mark.parametrize("n,k,m", [(80, 272, 3), (33, 1000, 5), (1, 16, 1), (300, 2048, 70)])
def test_ragged(n, k, m):
    (x, wq, ws), host = case(n, k, m, seed=95)
    check(qk.fp8w_gemm(x, wq, ws), oracle.fp8_weight_only_reference(*host), f"N={n} K={k} M={m}")


def test_method_end_to_end_and_graph():
    n, k = 4096, 2048
    g = torch.Generator().manual_seed(96)
    lin = LinearBase(k, n, bias=True, dtype=torch.bfloat16, device="cuda")
    lin.weight.data.copy_((torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16))
    lin.bias.data.copy_(torch.randn(n, generator=g).to(torch.bfloat16))
    wnp = lin.weight.detach().float().cpu().numpy()
    bnp = lin.bias.detach().float().cpu().numpy()
    method = Fp8WeightOnlyMethod(calibrate=False)
    method.process_weights(lin)
    lin.quant_method = method
    assert method.applies_to(lin)
    assert lin.fp8_weight.shape == (k, n) and lin.fp8_weight.dtype == torch.float8_e4m3fn
    assert lin.fp8_scale.shape == (1, n) and lin.weight.numel() == 0
    wq, ws = oracle.quantize_weight_fp8(wnp)
    np.testing.assert_array_equal(lin.fp8_weight.t().contiguous().view(torch.uint8).cpu().numpy(), wq)
    xs = torch.zeros(8, k, dtype=torch.bfloat16, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        lin(xs)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = lin(xs)
    for seed in (97, 98):
        xn = torch.randn(8, k, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
        xs.copy_(xn.cuda())
        graph.replay()
        torch.cuda.synchronize()
        check(out, oracle.fp8_weight_only_reference(xn.float().numpy(), wq, ws, bnp), f"graph {seed}")
