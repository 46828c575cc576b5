"""Activation prologues on the sm_100a library: RMSNorm and SiLU·up, standalone and fused
into the W8A16 GEMM that consumes them.

Bars:
* RMSNorm (qtts/layers/norm.py:49-76, 123-137): within one representable step of the
  reference's eager form run by torch on the same GPU for 16-bit outputs, and within a few
  ULP in fp32 -- the bar the reference sets for its own fused kernel (its
  tests/test_norm.py) -- and within one step of the float64 oracle.
* SiLU·up (qtts/layers/activation.py:147): equal bit for bit to torch's F.silu(gate) * up
  on the GPU, over every bf16 and fp16 gate value.
* Fused GEMM: equal bit for bit to the standalone prologue kernel followed by the plain
  GEMM with the same kernel variant (the prologue's elements come from one shared
  definition), and within the W8A16 tolerance of the oracle (max relative error 1e-2,
  every output within one bf16 rounding + 1e-3 max|ref|).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from conftest import require_b200
from qtts_b200 import _native as nat
from qtts_b200.quant import kernels as qk

pytestmark = pytest.mark.gpu

TORCH_DTYPE = {"bf16": torch.bfloat16, "fp16": torch.float16, "f32": torch.float32}


@pytest.fixture(scope="module", autouse=True)
def _device():
    require_b200()
    nat.device_status(reset=True)
    yield
    torch.cuda.synchronize()
    assert nat.device_status() == 0, "a kernel recorded a device-side failure"


def eager_rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """The reference's eager RMSNorm (qtts/layers/norm.py:123-137), run by torch."""
    x32 = x.to(torch.float32)
    variance = x32.pow(2).mean(-1, keepdim=True)
    x32 = x32 * torch.rsqrt(variance + eps)
    return (w.to(torch.float32) * x32).to(x.dtype)


def steps(a: torch.Tensor, b: torch.Tensor, name: str) -> np.ndarray:
    return oracle.float_steps(a.float().cpu().numpy(), b.float().cpu().numpy(), name)


def norm_rows(rows: int, width: int, dtype: torch.dtype, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, width, generator=g) * 3.0
    if rows > 2:
        x[1] = 0.0
        x[2] *= 1e-5
    w = 1.0 + 0.1 * torch.randn(width, generator=g)
    return x.to(dtype).cuda(), w.to(dtype).cuda()


@pytest.mark.parametrize("name", ["bf16", "fp16", "f32"])
@pytest.mark.parametrize("width", [128, 512, 1024, 2048, 1000, 999, 8192])
def test_rms_norm_against_reference_forms(name, width):
    dtype = TORCH_DTYPE[name]
    x, w = norm_rows(24, width, dtype, seed=200 + width)
    ours = qk.rms_norm(x, w, 1e-6)
    tol = 1 if name != "f32" else 4
    s_eager = steps(ours, eager_rms_norm(x, w, 1e-6), name)
    assert s_eager.max() <= tol, f"{s_eager.max()} steps from the eager form"
    truth = oracle.rms_norm_reference(x.float().cpu().numpy(), w.float().cpu().numpy(), 1e-6, name)
    s_truth = oracle.float_steps(ours.float().cpu().numpy(), truth, name)
    assert s_truth.max() <= tol, f"{s_truth.max()} steps from the float64 answer"
    assert torch.all(ours[1] == 0)


def test_rms_norm_strided_rows_and_in_place():
    x, w = norm_rows(8 * 5, 1024, torch.bfloat16, seed=210)
    x3 = x.view(8, 5, 1024)
    last = qk.rms_norm(x3[:, -1], w, 1e-6)  # rows 5*1024 elements apart
    assert torch.equal(last, qk.rms_norm(x3[:, -1].contiguous(), w, 1e-6))
    want = qk.rms_norm(x, w, 1e-6)
    y = x.clone()
    qk.rms_norm(y, w, 1e-6, out=y)
    assert torch.equal(y, want)


@pytest.mark.parametrize("name", ["bf16", "fp16"])
def test_silu_mul_equals_torch_for_every_gate(name):
    dtype = TORCH_DTYPE[name]
    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16)
    gate = bits.view(dtype).reshape(256, 256)
    g = torch.Generator().manual_seed(220)
    up = (torch.randn(256, 256, generator=g) * 2.0).to(dtype)
    gate_up = torch.cat([gate, up], dim=1).cuda()
    ours = qk.silu_mul(gate_up)
    theirs = F.silu(gate_up[:, :256]) * gate_up[:, 256:]
    nan = torch.isnan(theirs)
    assert torch.equal(torch.isnan(ours), nan)
    assert torch.equal(ours[~nan], theirs[~nan]), "SiLU·up differs from torch's kernels"
    # The oracle agrees wherever numpy's exp does not tie-break differently.
    fin = ~nan.cpu()
    ref = oracle.silu_mul_reference(gate.float().numpy(), up.float().numpy(), name)
    assert oracle.float_steps(ours.float().cpu().numpy()[fin.numpy()], ref[fin.numpy()], name).max() <= 1


def test_silu_mul_fp32_and_ragged():
    g = torch.Generator().manual_seed(221)
    for dtype, width in ((torch.float32, 1024), (torch.bfloat16, 999), (torch.float16, 3)):
        gate_up = (torch.randn(7, 2 * width, generator=g) * 5).to(dtype).cuda()
        ours = qk.silu_mul(gate_up)
        theirs = F.silu(gate_up[:, :width]) * gate_up[:, width:]
        assert torch.equal(ours, theirs), f"{dtype} width {width}"


# ------------------------------------------------------------------ fused into the GEMM


def gemm_case(n: int, k: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    q, s = oracle.quantize_weight_per_channel(w.numpy())
    return torch.from_numpy(q).cuda(), torch.from_numpy(s).to(torch.bfloat16).cuda(), q, s


def check_w8a16(out: torch.Tensor, x_after_prologue: np.ndarray, q, s, what: str) -> None:
    ref = oracle.w8a16_reference(x_after_prologue, q, oracle.bf16_round(s))
    got = out.float().cpu().numpy().astype(np.float64)
    err = oracle.rel_err(got, ref)
    assert err <= 1e-2, f"{what}: rel err {err:.3e}"
    bad = np.abs(got - ref) > np.abs(ref) * 2.0**-8 + 1e-3 * np.abs(ref).max()
    assert not bad.any(), f"{what}: {bad.sum()} outputs beyond one bf16 rounding"


VARIANTS = {
    "auto": nat.VARIANT_AUTO,
    "generic": nat.VARIANT_GENERIC,
    "skinny1": nat.variant_skinny(1),
    "skinny2": nat.variant_skinny(2),
    "skinny4_r2": nat.variant_skinny(4, 2),
    "skinny8": nat.variant_skinny(8),
    "stream": nat.variant_stream(0),
    "stream3": nat.variant_stream(3),
    "umma1": nat.variant_umma(1),
    "umma2": nat.variant_umma(2),
}


def _applies(variant: str, m: int) -> bool:
    return not (variant.startswith("stream") and m > 16)


@pytest.mark.parametrize("variant", sorted(VARIANTS))
@pytest.mark.parametrize("m", [1, 3, 8, 16, 40])
def test_rmsnorm_gemm_fused_equals_two_steps(variant, m):
    if not _applies(variant, m):
        pytest.skip("the whole-K kernel takes M <= 16")
    n, k = 4096, 2048
    wq, ws, q, s = gemm_case(n, k, seed=230)
    x, nw = norm_rows(m, k, torch.bfloat16, seed=231 + m)
    v = VARIANTS[variant]
    xn = qk.rms_norm(x, nw, 1e-6)
    try:
        two = qk.w8_gemm(xn, wq, ws, variant=v)
    except RuntimeError as exc:  # the variant does not take this shape: neither form may
        with pytest.raises(RuntimeError, match="inapplicable kernel variant"):
            qk.w8_gemm_rmsnorm(x, nw, 1e-6, wq, ws, variant=v)
        assert "inapplicable kernel variant" in str(exc)
        return
    fused = qk.w8_gemm_rmsnorm(x, nw, 1e-6, wq, ws, variant=v)
    assert torch.equal(fused, two), f"{variant} M={m}: fused and two-step forms differ"
    check_w8a16(fused, xn.float().cpu().numpy(), q, s, f"{variant} M={m}")


@pytest.mark.parametrize("variant", sorted(VARIANTS))
@pytest.mark.parametrize("m", [1, 4, 8, 16, 40])
def test_silu_mul_gemm_fused_equals_two_steps(variant, m):
    if not _applies(variant, m):
        pytest.skip("the whole-K kernel takes M <= 16")
    n, k = 2048, 6144
    wq, ws, q, s = gemm_case(n, k, seed=240)
    g = torch.Generator().manual_seed(241 + m)
    gate_up = (torch.randn(m, 2 * k, generator=g) * 2.0).to(torch.bfloat16).cuda()
    v = VARIANTS[variant]
    act = F.silu(gate_up[:, :k]) * gate_up[:, k:]
    try:
        two = qk.w8_gemm(act, wq, ws, variant=v)
    except RuntimeError as exc:  # the variant does not take this shape: neither form may
        with pytest.raises(RuntimeError, match="inapplicable kernel variant"):
            qk.w8_gemm_silu_mul(gate_up, wq, ws, variant=v)
        assert "inapplicable kernel variant" in str(exc)
        return
    fused = qk.w8_gemm_silu_mul(gate_up, wq, ws, variant=v)
    assert torch.equal(fused, two), f"{variant} M={m}: fused and two-step forms differ"
    check_w8a16(fused, act.float().cpu().numpy(), q, s, f"{variant} M={m}")


@pytest.mark.parametrize("m", [1, 8, 16, 64, 128])
def test_talker_shapes_auto(m):
    for n, k, which in ((12288, 2048, "rms"), (2048, 6144, "silu"), (3072, 2048, "rms"), (4096, 1024, "rms"),
                        (6144, 1024, "rms"), (1024, 3072, "silu")):
        wq, ws, q, s = gemm_case(n, k, seed=250 + n)
        if which == "rms":
            x, nw = norm_rows(m, k, torch.bfloat16, seed=251)
            out = qk.w8_gemm_rmsnorm(x, nw, 1e-6, wq, ws)
            act = qk.rms_norm(x, nw, 1e-6)
        else:
            x = torch.randn(m, 2 * k, generator=torch.Generator().manual_seed(252)).to(torch.bfloat16).cuda()
            out = qk.w8_gemm_silu_mul(x, wq, ws)
            act = qk.silu_mul(x)
        assert torch.equal(out, qk.w8_gemm(act, wq, ws)), f"N={n} K={k} M={m}"
        staged = nat.plan(m, n, k)["kernel"] in ("skinny_w8a16_kernel", "stream_w8a16_kernel")
        assert qk.prologue_fused(m, n, k, nat.PROLOGUE_RMSNORM) == staged


def test_fp16_bias_and_strided_rows():
    n, k, m = 1024, 1024, 5
    g = torch.Generator().manual_seed(260)
    w = torch.randn(n, k, generator=g) * 0.02
    q, s = oracle.quantize_weight_per_channel(w.numpy())
    wq, ws = torch.from_numpy(q).cuda(), torch.from_numpy(s).to(torch.float16).cuda()
    bias = torch.randn(n, generator=g).to(torch.float16).cuda()
    x3 = (torch.randn(m, 3, k, generator=g) * 2).to(torch.float16).cuda()
    nw = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.float16).cuda()
    fused = qk.w8_gemm_rmsnorm(x3[:, -1], nw, 1e-5, wq, ws, bias)
    two = qk.w8_gemm(qk.rms_norm(x3[:, -1].contiguous(), nw, 1e-5), wq, ws, bias)
    assert torch.equal(fused, two)


def test_refusals_through_the_c_abi():
    lib = nat.lib()
    n, k, m = 256, 256, 40
    wq, ws, _, _ = gemm_case(n, k, seed=270)
    x = torch.zeros(m, 2 * k, dtype=torch.bfloat16, device="cuda")
    nw = torch.ones(k, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    stream = nat.stream_ptr(x.device)

    def call(prologue, ldx, norm, workspace, rows=m):
        return lib.qtts_w8a16_gemm_prologue(
            x.data_ptr(), ldx, nat.BF16, prologue, norm, ctypes.c_float(1e-6), wq.data_ptr(), k, ws.data_ptr(),
            nat.BF16, None, out.data_ptr(), n, rows, n, k, workspace, nat.VARIANT_AUTO, 0, stream)

    assert call(nat.PROLOGUE_RMSNORM, 2 * k, nw.data_ptr(), None) == 1  # M = 40 needs a workspace
    assert call(9, 2 * k, nw.data_ptr(), None) == 7  # unknown prologue
    assert call(nat.PROLOGUE_SILU_MUL, k, None, None, rows=8) == 2  # [gate | up] needs ldx >= 2K
    assert call(nat.PROLOGUE_RMSNORM, 2 * k, None, None, rows=8) == 1  # no norm weight
    assert lib.qtts_rms_norm(x.data_ptr(), k - 1, nw.data_ptr(), out.data_ptr(), n, nat.BF16, 4, k,
                             ctypes.c_float(1e-6), 0, stream) == 2
    torch.cuda.synchronize()


@pytest.mark.parametrize("m", [8, 40])
def test_graph_replays(m):
    n, k = 4096, 2048
    wq, ws, _, _ = gemm_case(n, k, seed=280)
    _, nw = norm_rows(1, k, torch.bfloat16, seed=281)
    xs = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    gu = torch.zeros(m, 2 * 1024, dtype=torch.bfloat16, device="cuda")
    wd, wsd, _, _ = gemm_case(512, 1024, seed=282)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        qk.w8_gemm_rmsnorm(xs, nw, 1e-6, wq, ws)
        qk.w8_gemm_silu_mul(gu, wd, wsd)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y1 = qk.w8_gemm_rmsnorm(xs, nw, 1e-6, wq, ws)
        y2 = qk.w8_gemm_silu_mul(gu, wd, wsd)
    for seed in (283, 284):
        g = torch.Generator().manual_seed(seed)
        xs.copy_((torch.randn(m, k, generator=g) * 3).to(torch.bfloat16).cuda())
        gu.copy_((torch.randn(m, 2048, generator=g) * 2).to(torch.bfloat16).cuda())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y1, qk.w8_gemm(qk.rms_norm(xs, nw, 1e-6), wq, ws)), f"replay {seed}"
        assert torch.equal(y2, qk.w8_gemm(qk.silu_mul(gu), wd, wsd)), f"replay {seed}"


def test_rms_norm_paths_agree_bit_for_bit():
    """Rows read once into registers (aligned, <= 2048 wide) and rows read twice (here made
    unaligned by an odd row pitch) give the same bits: one fixed reduction order."""
    x, w = norm_rows(12, 2048, torch.bfloat16, seed=290)
    padded = torch.zeros(12, 2049, dtype=torch.bfloat16, device="cuda")
    padded[:, :2048] = x
    assert torch.equal(qk.rms_norm(padded[:, :2048], w, 1e-6), qk.rms_norm(x, w, 1e-6))


@pytest.mark.parametrize("m", [1, 4, 8, 16])
@pytest.mark.parametrize("variant", ["auto", "skinny8", "stream"])
def test_rmsnorm_gemm_full_row_form(m, variant):
    """K = 1152 is not a multiple of the norm's 256-column groups: the streaming kernels
    load the rows once more for the factor. Still equal to the two-step form."""
    n, k = 2048, 1152
    wq, ws, q, s = gemm_case(n, k, seed=291)
    x, nw = norm_rows(m, k, torch.bfloat16, seed=292 + m)
    v = VARIANTS[variant]
    xn = qk.rms_norm(x, nw, 1e-6)
    assert torch.equal(qk.w8_gemm_rmsnorm(x, nw, 1e-6, wq, ws, variant=v), qk.w8_gemm(xn, wq, ws, variant=v))
