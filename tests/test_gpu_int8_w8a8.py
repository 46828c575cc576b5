"""int8 W8A8 (Int8Method) on the sm_100a library, bit for bit against the reference.

The reference computes Int8Method.apply with torch ops and torch._int_mm
(qtts/quant/int8.py:120-155); the library replaces them with a per-token int8
quantization kernel and a tcgen05 kind::i8 GEMM whose int32 sums are exact and
whose epilogue repeats the reference's fp32 roundings. So the bar here is
equality: the activation codes and scales with the reference's op sequence
run by torch on the same GPU, and the outputs with the float64-free oracle
(int64 sums, fp32 products in the reference's order) and with the reference's
own expression on the GPU.
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
from qtts_b200.quant.int8 import Int8Method

pytestmark = pytest.mark.gpu

SHAPES = [("qkv", 4096, 2048), ("o_proj", 2048, 2048), ("gate_up", 12288, 2048), ("down_proj", 2048, 6144)]
TORCH_DTYPE = {"bf16": torch.bfloat16, "fp16": torch.float16, "f32": torch.float32}


@pytest.fixture(scope="module", autouse=True)
def _device():
    require_b200()
    nat.device_status(reset=True)
    yield
    torch.cuda.synchronize()
    assert nat.device_status() == 0, "a kernel recorded a device-side failure"


def reference_act_quant(flat: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's activation quantization (qtts/quant/int8.py:138-140), run by torch."""
    scale_x = flat.abs().amax(dim=1, keepdim=True).clamp_min(1e-6) / 127.0
    q = (flat / scale_x).round().clamp_(-127, 127).to(torch.int8)
    return q, scale_x


def test_quantizer_matches_reference_ops_on_gpu():
    g = torch.Generator().manual_seed(120)
    for name, dtype in TORCH_DTYPE.items():
        x = torch.randn(12, 1000, generator=g) * torch.logspace(-5, 3, 12)[:, None]
        x[1] = 0.0
        x[4, 7] = 900.0  # a single spike
        x = x.to(dtype).cuda()
        q_ref, s_ref = reference_act_quant(x)
        q, s = qk.int8_quant_rows(x)
        assert torch.equal(q, q_ref), f"{name}: int8 codes differ from the reference's ops"
        assert torch.equal(s, s_ref.float()), f"{name}: scales differ from the reference's ops"
        qo, so = oracle.quantize_act_int8(x.float().cpu().numpy(), name if name != "f32" else "f32")
        np.testing.assert_array_equal(q.cpu().numpy(), qo)
        np.testing.assert_array_equal(s.cpu().numpy().ravel(), so)


def case(n, k, m, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    x = torch.randn(m, k, generator=g).to(dtype)
    wq, ws = oracle.quantize_weight_per_channel(w.numpy())
    xq, xs = oracle.quantize_act_int8(x.float().numpy(), {torch.bfloat16: "bf16", torch.float16: "fp16",
                                                          torch.float32: "f32"}[dtype])
    return xq, xs, wq, ws


def check_exact(out, xq, xs, wq, ws, bias, dtype_name, what):
    ref = oracle.round_to(oracle.int8_w8a8_reference(xq, xs, wq, ws, bias), dtype_name)
    got = out.float().cpu().numpy()
    bad = got != ref
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outputs differ (max |d| {np.abs(got - ref).max():.3e})"


@pytest.mark.parametrize("label,n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 5, 16, 17, 64, 128, 200])
def test_gemm_bit_exact_on_talker_shapes(label, n, k, m):
    xq, xs, wq, ws = case(n, k, m, seed=121)
    out = qk.i8_scaled_mm(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), torch.from_numpy(wq).cuda(),
                          torch.from_numpy(ws).cuda(), None, torch.bfloat16)
    check_exact(out, xq, xs, wq, ws, None, "bf16", f"{label} M={m}")


VARIANTS = {"generic": nat.VARIANT_GENERIC, **{f"tc{s}": nat.variant_umma(s) for s in (1, 2, 4)}}


@pytest.mark.parametrize("variant", sorted(VARIANTS))
@pytest.mark.parametrize("m", [3, 40])
@pytest.mark.parametrize("out_dtype", ["bf16", "fp16", "f32"])
def test_variants_bias_and_output_types(variant, m, out_dtype):
    n, k = 1024, 2048
    xq, xs, wq, ws = case(n, k, m, seed=122)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(123)).to(TORCH_DTYPE[out_dtype])
    out = qk.i8_scaled_mm(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), torch.from_numpy(wq).cuda(),
                          torch.from_numpy(ws).cuda(), bias.cuda(), TORCH_DTYPE[out_dtype],
                          variant=VARIANTS[variant])
    assert out.dtype == TORCH_DTYPE[out_dtype]
    check_exact(out, xq, xs, wq, ws, bias.float().numpy(), out_dtype, f"{variant} M={m} {out_dtype}")


@pytest.mark.parametrize("n,k,m", [(80, 272, 3), (33, 1000, 5), (1, 16, 1), (300, 2048, 130), (7, 40, 2)])
def test_ragged_shapes(n, k, m):
    xq, xs, wq, ws = case(n, k, m, seed=124)
    out = qk.i8_scaled_mm(torch.from_numpy(xq).cuda(), torch.from_numpy(xs).cuda(), torch.from_numpy(wq).cuda(),
                          torch.from_numpy(ws).cuda(), None, torch.bfloat16)
    check_exact(out, xq, xs, wq, ws, None, "bf16", f"N={n} K={k} M={m}")


def test_large_sums_stay_exact():
    # All +-127 codes: |sum| reaches 127 * 127 * 6144 ~ 9.9e7 > 2^24, so an fp32
    # accumulator or fp32 split-K partials would round; the int32 path must not.
    n, k, m = 512, 6144, 16
    g = torch.Generator().manual_seed(125)
    wq = (torch.randint(0, 2, (n, k), generator=g) * 254 - 127).to(torch.int8)
    xq = (torch.randint(0, 2, (m, k), generator=g) * 254 - 127).to(torch.int8)
    wq[:8] = 127
    xq[:4] = 127
    xs = torch.full((m,), 1.0)
    ws = torch.full((n,), 1.0)
    for v in (nat.variant_umma(1), nat.variant_umma(4), nat.VARIANT_GENERIC):
        out = qk.i8_scaled_mm(xq.cuda(), xs.cuda(), wq.cuda(), ws.cuda(), None, torch.float32, variant=v)
        ref = oracle.int8_w8a8_reference(xq.numpy(), xs.numpy(), wq.numpy(), ws.numpy())
        np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_int8_method_matches_reference_apply_on_gpu(dtype):
    """Int8Method through LinearBase vs the reference's own apply expression on the GPU
    (torch ops, torch._int_mm with its 17-row padding): equal, in a CUDA graph too."""
    td = TORCH_DTYPE[dtype]
    n, k = 4096, 2048
    g = torch.Generator().manual_seed(126)
    lin = LinearBase(k, n, bias=True, dtype=td, device="cuda")
    lin.weight.data.copy_((torch.randn(n, k, generator=g) * 0.02).to(td))
    lin.bias.data.copy_(torch.randn(n, generator=g).to(td))
    w_ref = lin.weight.detach().float()
    method = Int8Method()
    method.process_weights(lin)
    lin.quant_method = method
    assert lin.int8_weight.shape == (k, n) and lin.int8_weight.dtype == torch.int8
    assert lin.int8_scale.dtype == torch.float32
    # The reference's weight quantization on the GPU (int8.py:45-56) gives the same codes.
    ref_scale = w_ref.abs().amax(dim=1).clamp_min(1e-12) / 127.0
    ref_q = (w_ref / ref_scale[:, None]).round().clamp_(-127, 127).to(torch.int8)
    assert torch.equal(lin.int8_weight.t(), ref_q) and torch.equal(lin.int8_scale, ref_scale)

    def reference_apply(x):
        q, scale_x = reference_act_quant(x)
        rows = q.shape[0]
        qp = torch.cat([q, q.new_zeros(max(0, 17 - rows), q.shape[1])], dim=0)
        acc = torch._int_mm(qp, ref_q.t().contiguous())[:rows]
        out = acc.float() * scale_x.float() * ref_scale.reshape(1, -1)
        out += lin.bias.float()
        return out.to(td)

    for m in (1, 8, 40):
        x = torch.randn(m, k, generator=g).to(td).cuda()
        assert torch.equal(lin(x), reference_apply(x)), f"M={m}"
    xs = torch.zeros(8, k, dtype=td, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        lin(xs)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = lin(xs)
    for seed in (127, 128):
        xs.copy_(torch.randn(8, k, generator=torch.Generator().manual_seed(seed)).to(td).cuda())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, reference_apply(xs)), f"graph replay {seed}"
