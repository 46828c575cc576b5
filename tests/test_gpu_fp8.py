"""Parity of the fp8-e4m3 path (quantizers + tcgen05 scaled GEMM) with the oracle, through the C ABI.

Integer outputs are bit-exact: e4m3 codes and fp32 scales of the weight and
activation quantizers (qtts/quant/fp8.py:45-49, 77-78), against the oracle's
CUDA form and against the reference's op sequence run by torch on the GPU. The GEMM multiplies
e4m3 values exactly in fp32, so its outputs are held within one output
rounding of the float64 value of the reference's math
(`_scaled_mm(q, W.t(), scale_a, scale_b) + bias`, fp8.py:79-88), and the whole
`Fp8Method` forward is also compared with the reference's own op sequence run
with torch on the GPU (`torch._scaled_mm`).
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
from qtts_b200.quant.fp8 import Fp8Method

pytestmark = pytest.mark.gpu

SHAPES = [("qkv", 4096, 2048), ("o_proj", 2048, 2048), ("gate_up", 12288, 2048), ("down_proj", 2048, 6144)]


@pytest.fixture(scope="module", autouse=True)
def _device():
    require_b200()
    nat.device_status(reset=True)
    yield
    torch.cuda.synchronize()
    assert nat.device_status() == 0, "a kernel recorded a device-side failure"


def codes(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.uint8).cpu().numpy()


def check_close(out, ref, what, dtype=torch.bfloat16):
    out = out.float().cpu().numpy().astype(np.float64)
    err = oracle.rel_err(out, ref)
    assert err <= 1e-2, f"{what}: rel err {err:.3e}"
    step = {torch.bfloat16: 2.0**-8, torch.float16: 2.0**-11, torch.float32: 2.0**-22}[dtype]
    bound = np.abs(ref) * step + 2e-3 * np.abs(ref).max() + 1e-30
    bad = np.abs(out - ref) > bound
    assert not bad.any(), f"{what}: {bad.sum()} elements beyond one output rounding (rel err {err:.3e})"


@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_weight_quantizer_bit_exact(golden, src):
    w = torch.from_numpy(golden[f"w_{src}"])
    if src == "bf16":
        w = w.to(torch.bfloat16)
    q, s = qk.quantize_fp8_rows(w.cuda())
    qo, so = oracle.quantize_weight_fp8(golden[f"w_{src}"], device="cuda")
    np.testing.assert_array_equal(codes(q), qo)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))
    same = so == golden[f"fp8_scale_{src}"]  # rows where the CPU-made golden scale agrees
    np.testing.assert_array_equal(codes(q)[same], golden[f"fp8_q_{src}"][same])


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "f32"])
def test_activation_quantizer_bit_exact(golden, dtype):
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "f32": torch.float32}[dtype]
    x = torch.from_numpy(golden[f"act_x_{dtype}"]).to(tdt).cuda()
    q, s = qk.fp8_quant_rows(x)
    qo, so = oracle.quantize_act_fp8(golden[f"act_x_{dtype}"], "fp32" if dtype == "f32" else dtype, device="cuda")
    np.testing.assert_array_equal(s.reshape(-1).cpu().numpy().view(np.uint32), so.view(np.uint32))
    np.testing.assert_array_equal(codes(q), qo)
    same = so == golden[f"act_scale_{dtype}"]
    np.testing.assert_array_equal(codes(q)[same], golden[f"act_q_{dtype}"][same])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_quantizers_match_reference_ops_on_gpu(dtype):
    """The reference's own op sequences (qtts/quant/fp8.py:45-49, 74-78), run by torch on the GPU."""
    g = torch.Generator().manual_seed(59)
    w = (torch.randn(4096, 2048, generator=g) * 0.02).to(dtype).cuda()
    wf = w.detach().float()
    ref_ws = wf.abs().amax(dim=1).clamp_min(1e-12) / 448.0
    ref_wq = (wf / ref_ws[:, None]).to(torch.float8_e4m3fn)
    q, s = qk.quantize_fp8_rows(w)
    assert torch.equal(s, ref_ws)
    assert torch.equal(q.view(torch.uint8), ref_wq.view(torch.uint8))
    qo, so = oracle.quantize_weight_fp8(wf.cpu().numpy(), device="cuda")
    np.testing.assert_array_equal(ref_ws.cpu().numpy(), so)
    np.testing.assert_array_equal(codes(ref_wq), qo)

    x = (torch.randn(64, 6144, generator=g) * torch.logspace(-8, 2, 64)[:, None]).to(dtype).cuda()
    x[5] = 0
    ref_sx = x.abs().amax(dim=1, keepdim=True).clamp_min(1e-6).float() / 448.0
    ref_xq = (x.float() / ref_sx).to(torch.float8_e4m3fn)
    xq, sx = qk.fp8_quant_rows(x)
    assert torch.equal(sx, ref_sx)
    assert torch.equal(xq.view(torch.uint8), ref_xq.view(torch.uint8))


def test_quantizers_full_size():
    g = torch.Generator().manual_seed(60)
    w = torch.randn(12288, 2048, generator=g) * 0.02
    q, s = qk.quantize_fp8_rows(w.cuda())
    qo, so = oracle.quantize_weight_fp8(w.numpy())
    np.testing.assert_array_equal(codes(q), qo)
    np.testing.assert_array_equal(s.cpu().numpy(), so)
    x = (torch.randn(100, 6144, generator=g) * torch.logspace(-9, 3, 100)[:, None]).to(torch.bfloat16)
    x[3] = 0
    qx, sx = qk.fp8_quant_rows(x.cuda())
    qxo, sxo = oracle.quantize_act_fp8(x.float().numpy(), "bf16")
    np.testing.assert_array_equal(sx.reshape(-1).cpu().numpy(), sxo)
    np.testing.assert_array_equal(codes(qx), qxo)


def fp8_case(n, k, m, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    wq, ws = oracle.quantize_weight_fp8(w.numpy())
    xq, xs = oracle.quantize_act_fp8(x.float().numpy(), "bf16")
    dev = lambda a, dt: torch.from_numpy(a).cuda().view(dt) if dt is not None else torch.from_numpy(a).cuda()
    return (dev(xq, torch.float8_e4m3fn), dev(xs, None), dev(wq, torch.float8_e4m3fn), dev(ws, None)), (xq, xs, wq, ws)


@pytest.mark.parametrize("label,n,k", SHAPES)
@pytest.mark.parametrize("m", [1, 16, 17, 32, 64, 100, 128, 200])
def test_scaled_gemm_talker_shapes(label, n, k, m):
    (xq, xs, wq, ws), host = fp8_case(n, k, m, seed=61)
    ref = oracle.fp8_scaled_mm_reference(*host)
    out = qk.fp8_scaled_mm(xq, xs, wq, ws, None, torch.bfloat16)
    check_close(out, ref, f"{label} M={m}")


@pytest.mark.parametrize("variant", ["generic", "tc1", "tc2", "tc4"])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_variants_dtypes_bias(variant, out_dtype):
    n, k, m = 2048, 6144, 24
    (xq, xs, wq, ws), host = fp8_case(n, k, m, seed=62)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(63))
    ref = oracle.fp8_scaled_mm_reference(*host, bias=bias.to(out_dtype).float().numpy())
    v = nat.VARIANT_GENERIC if variant == "generic" else nat.variant_umma(int(variant[-1]))
    out = qk.fp8_scaled_mm(xq, xs, wq, ws, bias.to(out_dtype).cuda(), out_dtype, variant=v)
    assert out.dtype == out_dtype
    check_close(out, ref, f"{variant} {out_dtype}", out_dtype)
    # The bias is added as the reference adds it: to the GEMM's output already rounded to the
    # output dtype, in that dtype (fp8.py:79-88) -- equal bit for bit to torch's add.
    plain = qk.fp8_scaled_mm(xq, xs, wq, ws, None, out_dtype, variant=v)
    assert torch.equal(out, plain + bias.to(out_dtype).cuda())


@pytest.mark.parametrize("n,k,m", [(80, 272, 3), (300, 2048, 130), (1, 16, 1), (33, 1000, 5)])
def test_ragged_shapes(n, k, m):
    (xq, xs, wq, ws), host = fp8_case(n, k, m, seed=64)
    ref = oracle.fp8_scaled_mm_reference(*host)
    out = qk.fp8_scaled_mm(xq, xs, wq, ws, None, torch.bfloat16)
    check_close(out, ref, f"N={n} K={k} M={m}")


def test_fp8_method_matches_reference_ops():
    """Fp8Method end to end vs the reference's own sequence on the GPU (fp8.py:73-89)."""
    n, k, m = 4096, 2048, 16
    g = torch.Generator().manual_seed(65)
    lin = LinearBase(k, n, bias=True, dtype=torch.bfloat16, device="cuda")
    lin.weight.data.copy_((torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16))
    lin.bias.data.copy_(torch.randn(n, generator=g).to(torch.bfloat16))
    w_ref = lin.weight.detach().clone()
    x = torch.randn(2, m // 2, k, generator=g).to(torch.bfloat16).cuda()

    # The reference's op sequence, verbatim semantics, on torch's GPU kernels.
    wf = w_ref.float()
    ws = wf.abs().amax(dim=1).clamp_min(1e-12) / 448.0
    wq = (wf / ws[:, None]).to(torch.float8_e4m3fn)
    flat = x.reshape(-1, k)
    sx = flat.abs().amax(dim=1, keepdim=True).clamp_min(1e-6).float() / 448.0
    xq = (flat.float() / sx).to(torch.float8_e4m3fn)
    ref = torch._scaled_mm(xq, wq.t(), scale_a=sx, scale_b=ws.reshape(1, -1), bias=None, out_dtype=torch.bfloat16)
    ref = (ref + lin.bias).reshape(2, m // 2, n)

    method = Fp8Method()
    method.process_weights(lin)
    lin.quant_method = method
    assert lin.fp8_weight.shape == (k, n) and lin.fp8_weight.dtype == torch.float8_e4m3fn
    assert lin.fp8_scale.shape == (1, n)
    assert torch.equal(lin.fp8_weight.t().contiguous().view(torch.uint8), wq.view(torch.uint8))
    out = lin(x)
    assert out.shape == (2, m // 2, n)
    assert oracle.rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy()) <= 1e-2


def test_fp8_linear_in_cuda_graph():
    n, k, m = 2048, 2048, 32
    g = torch.Generator().manual_seed(66)
    lin = LinearBase(k, n, dtype=torch.bfloat16, device="cuda")
    lin.weight.data.copy_((torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16))
    wnp = lin.weight.detach().float().cpu().numpy()
    method = Fp8Method()
    method.process_weights(lin)
    lin.quant_method = method
    xs = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        lin(xs)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = lin(xs)
    wq, wsc = oracle.quantize_weight_fp8(wnp)
    for seed in (67, 68):
        xn = torch.randn(m, k, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
        xs.copy_(xn.cuda())
        graph.replay()
        torch.cuda.synchronize()
        xq, sx = oracle.quantize_act_fp8(xn.float().numpy(), "bf16")
        ref = oracle.fp8_scaled_mm_reference(xq, sx, wq, wsc)
        check_close(out, ref, f"graph replay {seed}")
