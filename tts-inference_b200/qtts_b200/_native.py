"""ctypes binding of the C ABI in ``include/qtts_b200.h``.

The shared library is the product; this module only loads it and converts
torch tensors to the pointers, leading dimensions and dtype codes the ABI
takes. There is no fallback: when the library cannot be loaded every entry
point raises ``RuntimeError`` with the reason.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

from .build import LIB_PATH

# dtype codes (enum qtts_dtype)
BF16, FP16, FP32, E4M3, INT8 = 0, 1, 2, 3, 4

_TORCH_TO_CODE = {
    torch.bfloat16: BF16,
    torch.float16: FP16,
    torch.float32: FP32,
    torch.int8: INT8,
}
if hasattr(torch, "float8_e4m3fn"):
    _TORCH_TO_CODE[torch.float8_e4m3fn] = E4M3

# status codes (enum qtts_status)
OK = 0
ERR_TIMEOUT = 8

FLAG_PDL = 0x1
# activation prologues (QTTS_PROLOGUE_*)
PROLOGUE_NONE, PROLOGUE_RMSNORM, PROLOGUE_SILU_MUL = 0, 1, 2
VARIANT_AUTO = 0
VARIANT_GENERIC = 1


def variant_skinny(split: int, rows: int = 0) -> int:
    """Skinny kernel: K split over `split` clustered CTAs, `rows` row groups of 16 per CTA (0 = choose)."""
    return 0x100 | split | (rows << 4)


def variant_umma(split: int) -> int:
    return 0x200 | split


def variant_stream(rows: int = 0) -> int:
    """Weight-streaming kernel (M <= 16): 16*`rows` output rows per CTA (0 = choose)."""
    return 0x300 | (rows << 4)


# Every symbol the header declares, with its ctypes signature.
_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_vp = ctypes.c_void_p
_c_uint = ctypes.c_uint
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "qtts_abi_version": (_c_int, []),
    "qtts_status_str": (ctypes.c_char_p, [_c_int]),
    "qtts_device_status": (_c_int, [_c_int]),
    "qtts_set_wait_limit_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "qtts_w8a16_gemm": (
        _c_int,
        [_c_vp, _c_i64, _c_int, _c_vp, _c_i64, _c_vp, _c_int, _c_vp, _c_vp, _c_i64, _c_int, _c_int, _c_int,
         _c_int, _c_uint, _c_vp],
    ),
    "qtts_fp8w_gemm": (
        _c_int,
        [_c_vp, _c_i64, _c_int, _c_vp, _c_i64, _c_vp, _c_int, _c_vp, _c_vp, _c_i64, _c_int, _c_int, _c_int,
         _c_int, _c_uint, _c_vp],
    ),
    "qtts_int8_quant_rows": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_int, _c_uint, _c_vp]),
    "qtts_i8_gemm": (
        _c_int,
        [_c_vp, _c_i64, _c_vp, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_uint, _c_vp],
    ),
    "qtts_w8a16_plan": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp, _c_vp]),
    "qtts_w8a16_gemm_allgather": (
        _c_int,
        [_c_vp, _c_i64, _c_int, _c_vp, _c_i64, _c_vp, _c_int, _c_vp, _c_vp, _c_i64, _c_i64, _c_vp, _c_vp, _c_int,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_uint, _c_vp],
    ),
    "qtts_w8a16_grouped_gemm": (
        _c_int,
        [_c_vp, _c_i64, _c_i64, _c_int, _c_vp, _c_i64, _c_vp, _c_int, _c_vp, _c_vp, _c_i64, _c_i64, _c_int, _c_int,
         _c_int, _c_int, _c_vp, _c_int, _c_uint, _c_vp],
    ),
    "qtts_quantize_int8_rows": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_int, _c_vp]),
    "qtts_quantize_fp8_rows": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_int, _c_vp]),
    "qtts_fp8_quant_rows": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, _c_vp, _c_int, _c_int, _c_uint, _c_vp]),
    "qtts_fp8_gemm": (
        _c_int,
        [_c_vp, _c_i64, _c_vp, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_int, _c_int, _c_int, _c_int,
         _c_int, _c_uint, _c_vp],
    ),
    "qtts_rms_norm": (_c_int, [_c_vp, _c_i64, _c_vp, _c_vp, _c_i64, _c_int, _c_int, _c_int, ctypes.c_float,
                               _c_uint, _c_vp]),
    "qtts_silu_mul": (_c_int, [_c_vp, _c_i64, _c_vp, _c_i64, _c_int, _c_int, _c_int, _c_uint, _c_vp]),
    "qtts_w8a16_head_argmax": (_c_int, [_c_vp, _c_i64, _c_int, _c_vp, ctypes.c_float, _c_vp, _c_i64, _c_vp, _c_int,
                                        _c_vp, _c_vp, _c_vp, _c_i64, _c_int, _c_vp, _c_i64, _c_int, _c_vp, _c_int,
                                        _c_int, _c_int, _c_uint, _c_vp]),
    "qtts_w8a16_gemm_prologue": (
        _c_int,
        [_c_vp, _c_i64, _c_int, _c_int, _c_vp, ctypes.c_float, _c_vp, _c_i64, _c_vp, _c_int, _c_vp, _c_vp, _c_i64,
         _c_int, _c_int, _c_int, _c_vp, _c_int, _c_uint, _c_vp],
    ),
    "qtts_w8a16_gemm_prologue_fused": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "qtts_fp8_linear_noalloc": (
        _c_int,
        [_c_vp, _c_i64, _c_int, _c_vp, _c_i64, _c_vp, _c_vp, _c_vp, _c_i64, _c_int, _c_int, _c_int, _c_int,
         _c_uint, _c_vp],
    ),
}

_lib: ctypes.CDLL | None = None
_load_error: str | None = None
_lock = threading.Lock()


def _load() -> ctypes.CDLL:
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(LIB_PATH)
        if not path.exists():
            # Compile from source once if the library was never built here
            # (nvcc ships with the image). Still no fallback if that fails.
            try:
                from .build import build

                build()
            except Exception as exc:  # pragma: no cover - depends on the toolchain
                _load_error = f"{path} missing and the build failed: {exc}"
                raise RuntimeError(_load_error) from exc
        try:
            lib = ctypes.CDLL(str(path))
        except OSError as exc:
            _load_error = f"cannot load {path}: {exc}"
            raise RuntimeError(_load_error) from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _load()


def library_path() -> str:
    return str(LIB_PATH)


def available() -> tuple[bool, str]:
    """(True, "") when the library loads and a compute-capability 10.x GPU is visible."""
    try:
        _load()
    except RuntimeError as exc:
        return False, str(exc)
    if not torch.cuda.is_available():
        return False, "no CUDA device"
    major, minor = torch.cuda.get_device_capability()
    if major != 10:
        return False, f"compute capability {major}.{minor}: these kernels are built for sm_100a (B200) only"
    return True, ""


def status_str(code: int) -> str:
    return _load().qtts_status_str(code).decode()


def check(code: int, what: str) -> None:
    if code != OK:
        raise RuntimeError(f"{what} failed: {status_str(code)} (status {code})")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _TORCH_TO_CODE[dtype]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype {dtype}") from exc


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(reset: bool = False) -> int:
    return _load().qtts_device_status(1 if reset else 0)


def set_wait_limit_ns(limit_ns: int) -> int:
    return int(_load().qtts_set_wait_limit_ns(limit_ns))


KERNEL_NAMES = {0: "generic_w8a16_kernel", 1: "skinny_w8a16_kernel", 2: "umma_w8a16_kernel", 3: "stream_w8a16_kernel"}


def plan(m: int, n: int, k: int, groups: int = 1, variant: int = VARIANT_AUTO) -> dict:
    """The kernel and launch shape qtts_w8a16_gemm picks (host-only; no GPU needed)."""
    out = [ctypes.c_int() for _ in range(4)]
    check(lib().qtts_w8a16_plan(m, n, k, groups, variant, *[ctypes.byref(v) for v in out]), "qtts_w8a16_plan")
    kern, split, rows, ctas = (v.value for v in out)
    return {"kernel": KERNEL_NAMES[kern], "split": split, "row_tile": rows, "ctas": ctas}
