"""Pin the CPU oracle to the reference: golden vectors made by the reference's own code.

The vectors come from tests/golden/make_golden.py, which runs the reference's
``qtts.quant`` functions and tuning script on the CPU, so the quantizers are
checked here in their ``device="cpu"`` form (IEEE ``tensor / number``). Integer and e4m3 outputs and fp32
scales must match bit for bit; the eager bf16 GEMM within one bf16 rounding
step (its fp32 summation order is the BLAS library's).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle


@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_int8_quantizer_bit_exact(golden, src):
    q, s = oracle.quantize_weight_per_channel(golden[f"w_{src}"], device="cpu")
    np.testing.assert_array_equal(q, golden[f"int8_q_{src}"])
    np.testing.assert_array_equal(s.view(np.uint32), golden[f"int8_scale_{src}"].view(np.uint32))


def test_int8_quantizer_zero_row_floor(golden):
    q, s = oracle.quantize_weight_per_channel(golden["w_f32"], device="cpu")
    assert s[7] == np.float32(1e-12) / np.float32(127.0)
    assert not q[7].any()


@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_fp8_weight_quantizer_bit_exact(golden, src):
    q, s = oracle.quantize_weight_fp8(golden[f"w_{src}"], device="cpu")
    np.testing.assert_array_equal(q, golden[f"fp8_q_{src}"])
    np.testing.assert_array_equal(s.view(np.uint32), golden[f"fp8_scale_{src}"].view(np.uint32))


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "f32"])
def test_fp8_activation_quantizer_bit_exact(golden, dtype):
    x = golden[f"act_x_{dtype}"]
    q, s = oracle.quantize_act_fp8(x, "fp32" if dtype == "f32" else dtype, device="cpu")
    np.testing.assert_array_equal(s.view(np.uint32), golden[f"act_scale_{dtype}"].view(np.uint32))
    np.testing.assert_array_equal(q, golden[f"act_q_{dtype}"])


def test_tune_quantizer_bit_exact(golden):
    q, s = oracle.tune_quantize(golden["tune_w"], device="cpu")
    np.testing.assert_array_equal(q, golden["tune_q"])
    np.testing.assert_array_equal(s.view(np.uint32), golden["tune_scale"].view(np.uint32))


@pytest.mark.parametrize("m", [1, 3, 8])
def test_naive_dequant_linear(golden, m):
    y = oracle.naive_dequant_linear(golden[f"naive_x_m{m}"], golden["tune_q"], golden["tune_scale"])
    ref = golden[f"naive_y_m{m}"]
    # one bf16 step (2^-8 relative) of headroom for the BLAS summation order
    np.testing.assert_allclose(y, ref, rtol=2.0**-7, atol=1e-6)
    # and the fused-kernel math in float64 is within the reference's own error bar
    exact = oracle.w8a16_reference(golden[f"naive_x_m{m}"], golden["tune_q"], golden["tune_scale"])
    assert oracle.rel_err(ref, exact) < 1e-2


def test_e4m3_table_round_trip():
    codes = np.arange(256, dtype=np.uint8)
    vals = oracle.e4m3_decode(codes)
    finite = ~np.isnan(vals)
    np.testing.assert_array_equal(oracle.e4m3_encode(vals[finite]), codes[finite])
    assert np.nanmax(vals) == 448.0
    assert oracle.e4m3_decode(np.array([1], dtype=np.uint8))[0] == 2.0**-9


def test_e4m3_ties_round_to_even():
    # 1 + 1/16 lies halfway between 1 (code 0x38, even) and 1.125 (0x39, odd)
    assert oracle.e4m3_encode(np.array([1.0625], dtype=np.float32))[0] == 0x38
    # 1.1875 is halfway between 1.125 (0x39) and 1.25 (0x3A, even)
    assert oracle.e4m3_encode(np.array([1.1875], dtype=np.float32))[0] == 0x3A
    assert oracle.e4m3_encode(np.array([-1.1875], dtype=np.float32))[0] == 0xBA


def test_e4m3_matches_torch_cast():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    v = np.concatenate(
        [rng.standard_normal(4096) * s for s in (1e-4, 1e-2, 1.0, 30.0, 200.0)]
        + [np.array([0.0, -0.0, 448.0, -448.0, 2.0**-10, 3 * 2.0**-10, 447.9, 463.0])]
    ).astype(np.float32)
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(oracle.e4m3_encode(v), ref)


def test_bf16_round_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(2)
    v = (rng.standard_normal(10000) * 10.0 ** rng.integers(-8, 8, 10000)).astype(np.float32)
    ref = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(oracle.bf16_round(v), ref)


def test_rel_err_metric():
    assert oracle.rel_err(np.array([1.0, 2.0]), np.array([1.0, 2.0])) == 0.0
    assert oracle.rel_err(np.array([1.0, 2.5]), np.array([1.0, 2.0])) == pytest.approx(0.25)


def test_cuda_scalar_division_rule():
    """``device="cuda"`` differs from the CPU form only through ``a * fl32(1/c)``."""
    a = np.random.default_rng(7).random(100000, dtype=np.float32) * 4
    cpu = oracle.div_by_number(a, 448.0, "cpu")
    cuda = oracle.div_by_number(a, 448.0, "cuda")
    np.testing.assert_array_equal(cpu, a / np.float32(448))
    np.testing.assert_array_equal(cuda, a * (np.float32(1) / np.float32(448)))
    differ = (cpu != cuda).mean()
    assert 0 < differ < 1  # last-bit differences, on part of the inputs
    assert np.abs(cpu.view(np.int32) - cuda.view(np.int32)).max() == 1
    with pytest.raises(ValueError):
        oracle.div_by_number(a, 2.0, "mps")


@pytest.mark.parametrize("src", ["f32", "bf16"])
def test_quantizers_cuda_form_consistent(golden, src):
    """The CUDA-form quantizers agree with the CPU form wherever the scales agree."""
    w = golden[f"w_{src}"]
    for fn in (oracle.quantize_weight_per_channel, oracle.quantize_weight_fp8):
        qc, sc = fn(w, device="cpu")
        qg, sg = fn(w, device="cuda")
        same = sc == sg
        np.testing.assert_array_equal(qc[same], qg[same])
        assert np.all(np.abs(sc.view(np.int32) - sg.view(np.int32)) <= 1)


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "f32"])
def test_int8_w8a8_matches_reference(golden, dtype):
    """Int8Method (W8A8) through the oracle against the reference run on the CPU: the
    weight codes, the activation codes captured from torch._int_mm, and the output,
    bit for bit (the CPU form of ``tensor / number``)."""
    name = {"bf16": "bf16", "fp16": "fp16", "f32": "f32"}[dtype]
    w = oracle.round_to(golden["w8a8_w"], dtype)
    wq, ws = oracle.quantize_weight_per_channel(w, device="cpu")
    np.testing.assert_array_equal(wq, golden[f"w8a8_wq_{name}"])
    np.testing.assert_array_equal(ws, golden[f"w8a8_ws_{name}"])
    x = golden[f"w8a8_x_{name}"]
    q, sx = oracle.quantize_act_int8(x, dtype, device="cpu")
    np.testing.assert_array_equal(q, golden[f"w8a8_q_{name}"])
    bias = oracle.round_to(golden["w8a8_bias"], dtype)
    y = oracle.round_to(oracle.int8_w8a8_reference(q, sx, wq, ws, bias), dtype)
    np.testing.assert_array_equal(y, golden[f"w8a8_y_{name}"])


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "f32"])
@pytest.mark.parametrize("width", [128, 1024, 2048])
def test_rms_norm_matches_reference(golden, dtype, width):
    """RMSNorm through the oracle (float64, rounded once) against the reference's eager
    RMSNorm run on the CPU: within one representable step for 16-bit outputs (the bar the
    reference sets for its own fused kernel, tests/test_norm.py:55-72) and within a few
    ULP in fp32 (its fp32 bar), including an all-zero row and a row under the eps floor."""
    x, w, y = golden[f"rms_x_{dtype}_{width}"], golden[f"rms_w_{dtype}_{width}"], golden[f"rms_y_{dtype}_{width}"]
    ref = oracle.rms_norm_reference(x, w, 1e-6, dtype)
    steps = oracle.float_steps(ref, y, dtype)
    assert steps.max() <= (1 if dtype != "f32" else 4), f"{steps.max()} steps"
    assert np.all(y[1] == 0) and np.all(ref[1] == 0)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_silu_mul_matches_reference(golden, dtype):
    """F.silu(gate) * up through the oracle against the reference's expression run on the
    CPU, bit for bit, including zeros, saturating gates and tiny gates."""
    gu, y = golden[f"silu_gate_up_{dtype}"], golden[f"silu_y_{dtype}"]
    w = gu.shape[1] // 2
    np.testing.assert_array_equal(oracle.silu_mul_reference(gu[:, :w], gu[:, w:], dtype), y)


def test_float_steps_counts_representable_values():
    a = np.array([1.0, -1.0, 0.0, 1.0], dtype=np.float32)
    b = oracle.bf16_round(np.array([1.0078125, -1.0078125, -0.0, 1.0], dtype=np.float32))
    np.testing.assert_array_equal(oracle.float_steps(a, b, "bf16"), [1, 1, 0, 0])
