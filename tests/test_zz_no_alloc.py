"""qtts_fp8_linear_noalloc against the two-step fp8 sequence it stands for, through the C ABI.

The entry point keeps the activation codes and row scales in the library's own
device array; its outputs must equal those of qtts_fp8_quant_rows +
qtts_fp8_gemm with caller-provided buffers, call after call. Named to be
collected last, so it also runs after every other GPU test in one process.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import require_b200
from qtts_b200 import _native as nat

pytestmark = pytest.mark.gpu

MAX_ROWS = 1024
MAX_CODES = 1 << 20


@pytest.fixture(scope="module", autouse=True)
def _device():
    require_b200()
    nat.device_status(reset=True)
    yield
    torch.cuda.synchronize()
    assert nat.device_status() == 0


def weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    wq, ws = oracle.quantize_weight_fp8(w.numpy())
    return torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda()


def two_step(x, wq, ws, bias, out_dtype):
    """The existing entry points with torch-allocated scratch."""
    lib = nat.lib()
    m, k = x.shape
    n = wq.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    xq = torch.empty(m, k, dtype=torch.uint8, device="cuda")
    sx = torch.empty(m, dtype=torch.float32, device="cuda")
    nat.check(lib.qtts_fp8_quant_rows(x.data_ptr(), x.stride(0), nat.dtype_code(x.dtype), xq.data_ptr(),
                                      sx.data_ptr(), m, k, 1, stream), "qtts_fp8_quant_rows")
    out = torch.empty(m, n, dtype=out_dtype, device="cuda")
    nat.check(lib.qtts_fp8_gemm(xq.data_ptr(), k, sx.data_ptr(), wq.data_ptr(), wq.stride(0), ws.data_ptr(),
                                bias.data_ptr() if bias is not None else None, out.data_ptr(), n,
                                nat.dtype_code(out_dtype), m, n, k, 0, 1, stream), "qtts_fp8_gemm")
    return out


def no_alloc(x, wq, ws, bias, out):
    m, k = x.shape
    n = wq.shape[0]
    return nat.lib().qtts_fp8_linear_noalloc(
        x.data_ptr(), x.stride(0), nat.dtype_code(x.dtype), wq.data_ptr(), wq.stride(0), ws.data_ptr(),
        bias.data_ptr() if bias is not None else None, out.data_ptr(), out.stride(0), nat.dtype_code(out.dtype),
        m, n, k, 1, torch.cuda.current_stream().cuda_stream,
    )


@pytest.mark.parametrize(
    "m,n,k,out_dtype,with_bias",
    [
        (16, 4096, 2048, torch.bfloat16, False),   # talker qkv, tcgen05 GEMM
        (64, 2048, 6144, torch.bfloat16, True),    # talker down_proj
        (5, 300, 1000, torch.float16, True),       # K not a multiple of 16: SIMT GEMM
        (MAX_ROWS, 256, MAX_CODES // MAX_ROWS, torch.float32, False),  # the array exactly full
    ],
)
def test_matches_two_step_sequence(m, n, k, out_dtype, with_bias):
    wq, ws = weights(n, k, seed=70)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(71)).to(out_dtype).cuda() if with_bias else None
    out = torch.full((m, n), 7.0, dtype=out_dtype, device="cuda")
    for call, seed in enumerate((72, 73)):  # two calls in a row, different activations
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16).cuda()
        assert no_alloc(x, wq, ws, bias, out) == 0
        ref = two_step(x, wq, ws, bias, out_dtype)
        torch.cuda.synchronize()
        err = oracle.rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy())
        assert err <= 1e-2, f"call {call}: rel err {err:.3e}"
        assert torch.equal(out, ref), f"call {call}: outputs differ from the two-step sequence"


def test_rejects_problems_beyond_the_array():
    k = 2048
    wq, ws = weights(64, k, seed=74)
    for m in (MAX_CODES // k + 1, MAX_ROWS + 1):
        x = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
        out = torch.full((m, 64), 3.0, dtype=torch.bfloat16, device="cuda")
        code = no_alloc(x, wq, ws, None, out)
        assert code == 2 and "out of range" in nat.status_str(code)
        torch.cuda.synchronize()
        assert out.eq(3.0).all()
    m = MAX_ROWS + 1
    x = torch.zeros(m, 16, dtype=torch.bfloat16, device="cuda")
    wq16, ws16 = weights(64, 16, seed=75)
    out = torch.empty(m, 64, dtype=torch.bfloat16, device="cuda")
    assert no_alloc(x, wq16, ws16, None, out) == 2  # row limit, though M * K fits
