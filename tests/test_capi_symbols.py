"""The C-ABI library loads, exports every symbol the header declares, and validates
its arguments on the host before touching a device (no compute calls here)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from qtts_b200 import _native as nat
from qtts_b200.build import LIB_PATH

HEADER = Path(__file__).resolve().parents[1] / "include" / "qtts_b200.h"


def header_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"QTTS_API\s+[\w\s\*]+?\b(qtts_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    return nat.lib()


def test_library_file_is_in_tree():
    assert LIB_PATH.exists(), "build the library first (python -m qtts_b200.build)"
    assert "tts-inference_b200" in str(LIB_PATH)


def test_every_declared_symbol_is_exported(lib):
    declared = header_symbols()
    assert len(declared) >= 10
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} declared in qtts_b200.h but not exported"


def test_binding_covers_the_header():
    assert set(nat.SIGNATURES) == header_symbols()


def test_version_and_status_strings(lib):
    assert lib.qtts_abi_version() == 1
    assert nat.status_str(0) == "ok"
    for code in range(1, 10):
        assert nat.status_str(code) not in ("ok", "unknown status")
    assert nat.status_str(1234) == "unknown status"


def _w8a16(lib, *, x=16, w=16, scale=16, out=16, M=4, N=64, K=128, ldx=None, ldw=None, ldo=None,
           x_dtype=nat.BF16, scale_dtype=nat.BF16, variant=0):
    return lib.qtts_w8a16_gemm(
        x, ldx if ldx is not None else K, x_dtype, w, ldw if ldw is not None else K, scale, scale_dtype, None,
        out, ldo if ldo is not None else N, M, N, K, variant, 0, None,
    )


def test_host_validation_rejects_before_launch(lib):
    assert _w8a16(lib, M=-1) == 2  # QTTS_ERR_SHAPE
    assert _w8a16(lib, K=-5) == 2
    assert _w8a16(lib, x=None) == 1  # QTTS_ERR_NULL
    assert _w8a16(lib, scale=None) == 1
    assert _w8a16(lib, x_dtype=7) == 4  # QTTS_ERR_DTYPE
    assert _w8a16(lib, scale_dtype=nat.INT8) == 4
    assert _w8a16(lib, ldx=64) == 2  # ldx < K
    assert _w8a16(lib, ldo=8) == 2  # ldo < N


def test_empty_problem_is_a_noop(lib):
    assert _w8a16(lib, M=0, x=None, w=None, scale=None, out=None) == 0
    assert _w8a16(lib, N=0, x=None, w=None, scale=None, out=None) == 0


def test_no_device_reports_arch_error(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _w8a16(lib) == 5  # QTTS_ERR_ARCH: valid arguments, no sm_100 device


def test_noalloc_error_order(lib):
    """The scratch-free fp8 linear validates like the others: argument errors first, then
    QTTS_ERR_ARCH on a machine without an sm_100 device (before its scratch look-up)."""
    import torch

    def call(x=16, wq=16, sw=16, out=16, M=4, N=64, K=128, x_dtype=nat.BF16):
        return lib.qtts_fp8_linear_noalloc(x, K, x_dtype, wq, K, sw, None, out, N, nat.BF16, M, N, K, 0, None)

    assert call(M=-1) == 2
    assert call(x=None) == 1
    assert call(x_dtype=nat.INT8) == 4
    assert call(M=1025) == 2  # beyond QTTS_NOALLOC_MAX_ROWS
    assert call(M=1024, K=1025) == 2  # beyond QTTS_NOALLOC_MAX_CODES
    assert call(M=0, x=None) == 0
    if not torch.cuda.is_available():
        assert call() == 5  # QTTS_ERR_ARCH, not a CUDA error from the symbol look-up


def test_other_entry_points_validate(lib):
    assert lib.qtts_fp8_quant_rows(None, 16, nat.BF16, 16, 16, 2, 16, 0, None) == 1
    assert lib.qtts_fp8_quant_rows(16, 8, nat.BF16, 16, 16, 2, 16, 0, None) == 2
    assert lib.qtts_fp8_gemm(16, 16, 16, 16, 16, 16, None, 16, 16, nat.INT8, 2, 2, 16, 0, 0, None) == 4
    assert lib.qtts_quantize_int8_rows(16, 16, 9, 16, 16, 4, 16, None) in (4, 5)
    assert lib.qtts_quantize_fp8_rows(None, 16, nat.BF16, 16, 16, 4, 16, None) == 1
    assert lib.qtts_w8a16_grouped_gemm(16, 0, 16, nat.BF16, 16, 16, 16, nat.BF16, None, 16, 0, 16,
                                       0, 1, 1, 16, None, 0, 0, None) == 2  # G < 1


def test_wait_limit_roundtrip(lib):
    prev = nat.set_wait_limit_ns(123456789)
    assert nat.set_wait_limit_ns(0) == 123456789
    assert nat.set_wait_limit_ns(prev) == 2_000_000_000


def test_library_has_no_torch_dependency():
    # The ABI boundary is plain C: the shared object must not link libtorch.
    import subprocess

    out = subprocess.run(["ldd", str(LIB_PATH)], capture_output=True, text=True).stdout
    assert "torch" not in out and "libc10" not in out
    assert ctypes.CDLL(str(LIB_PATH)).qtts_abi_version() == 1


def test_prologue_entry_points_validate(lib):
    """The activation prologues reject bad arguments on the host, before any device call
    (so no GPU is needed to see it); valid arguments reach the device check."""
    bf16, f1 = nat.BF16, ctypes.c_float(1e-6)
    # qtts_rms_norm(x, ldx, weight, out, ldo, dtype, rows, width, eps, flags, stream)
    assert lib.qtts_rms_norm(16, 64, 16, 16, 64, bf16, -1, 64, f1, 0, None) == 2
    assert lib.qtts_rms_norm(16, 64, 16, 16, 64, bf16, 0, 64, f1, 0, None) == 0  # no rows: no-op
    assert lib.qtts_rms_norm(None, 64, 16, 16, 64, bf16, 4, 64, f1, 0, None) == 1
    assert lib.qtts_rms_norm(16, 32, 16, 16, 64, bf16, 4, 64, f1, 0, None) == 2  # ldx < width
    assert lib.qtts_rms_norm(16, 1 << 17, 16, 16, 1 << 17, bf16, 4, 65544, f1, 0, None) == 2  # too wide
    assert lib.qtts_rms_norm(16, 64, 16, 16, 64, 9, 4, 64, f1, 0, None) == 4
    assert lib.qtts_rms_norm(16, 64, 16, 16, 64, bf16, 4, 64, f1, 0, None) == 5  # no sm_100 device
    # qtts_silu_mul(gate_up, ld_in, out, ldo, dtype, rows, width, flags, stream)
    assert lib.qtts_silu_mul(16, 64, 16, 64, bf16, 4, 64, 0, None) == 2  # ld_in < 2 * width
    assert lib.qtts_silu_mul(None, 128, 16, 64, bf16, 4, 64, 0, None) == 1
    assert lib.qtts_silu_mul(16, 128, 16, 64, bf16, 4, 64, 0, None) == 5

    # qtts_w8a16_gemm_prologue(x, ldx, x_dtype, prologue, norm_weight, eps, w, ldw, scale,
    #   scale_dtype, bias, out, ldo, M, N, K, workspace, variant, flags, stream)
    def call(prologue=nat.PROLOGUE_RMSNORM, ldx=256, norm=16, m=8, variant=0, workspace=None):
        return lib.qtts_w8a16_gemm_prologue(16, ldx, bf16, prologue, norm, f1, 16, 256, 16, bf16, None, 16, 128,
                                            m, 128, 256, workspace, variant, 0, None)

    assert call(prologue=9) == 7
    assert call(norm=None) == 1
    assert call(prologue=nat.PROLOGUE_SILU_MUL, ldx=256) == 2  # [gate | up] rows need ldx >= 2K
    assert call(m=0) == 0
    assert call(m=40) == 1  # not fused at M > 16: the workspace is required
    assert call(m=40, workspace=16) == 5  # chained form, valid: reaches the device check
    assert call() == 5  # fused form, valid
