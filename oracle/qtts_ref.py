"""numpy restatement of the reference's quantized-linear arithmetic (test oracle).

TEST INFRASTRUCTURE ONLY -- imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the library.

Every function names the reference lines it restates (paths relative to the
danielhua23/tts-inference checkout). Floating-point steps are done in the
precision the reference uses, so integer outputs (int8 codes, e4m3 codes) and
fp32 scales are bit-exact, and GEMM outputs are computed in float64 as the
exact value the fp32-accumulating kernels approximate.
"""

from __future__ import annotations

import numpy as np

_F32 = np.float32

# ----------------------------------------------------------------------------
# 16-bit and 8-bit float formats


def bf16_round(a) -> np.ndarray:
    """float32 -> nearest bf16 (round half to even), returned as float32 values."""
    a = np.asarray(a, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32)
    return np.where(np.isnan(a), a, out).astype(np.float32)


def fp16_round(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(a, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_round(a)
    if dtype == "fp16":
        return fp16_round(a)
    return np.asarray(a, dtype=np.float32)


def _e4m3_table() -> np.ndarray:
    """Value of every float8_e4m3fn code: 1 sign, 4 exponent (bias 7), 3 mantissa bits,
    subnormals at exponent 0, no infinities, S.1111.111 is NaN."""
    vals = np.zeros(256, dtype=np.float64)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            vals[code] = np.nan
        elif e == 0:
            vals[code] = s * (m / 8.0) * 2.0**-6
        else:
            vals[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


_E4M3 = _e4m3_table()
_E4M3_POS = _E4M3[:127]  # codes 0..126: 0 .. 448 ascending


def e4m3_decode(codes) -> np.ndarray:
    return _E4M3[np.asarray(codes, dtype=np.uint8)].astype(np.float32)


def e4m3_encode(v) -> np.ndarray:
    """float32 -> float8_e4m3fn codes, round to nearest even.

    Magnitudes of 464 and above (half-way to the NaN code and beyond) give NaN,
    as torch's non-saturating cast does; the quantizers never produce them.
    """
    v = np.asarray(v, dtype=np.float32).astype(np.float64)
    mag = np.abs(v)
    hi = np.clip(np.searchsorted(_E4M3_POS, mag, side="left"), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    d_hi = np.abs(_E4M3_POS[hi] - mag)
    d_lo = np.abs(mag - _E4M3_POS[lo])
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(mag >= 464.0, np.uint8(0x7F), code)
    code = np.where(np.isnan(mag), np.uint8(0x7F), code)
    sign = np.signbit(v).astype(np.uint8) << 7
    return (code | sign).astype(np.uint8)


# ----------------------------------------------------------------------------
# Weight quantizers
#
# The reference divides a tensor by a Python number in three places (``amax /
# 127``, ``amax / 448``, ``scale / 448``). torch evaluates that differently by
# device: on the CPU it is an IEEE fp32 division; on a CUDA tensor the
# divisor is a CPU scalar, and torch multiplies by its reciprocal instead,
# ``a * fl32(1 / c)`` in the op's math type (fp32 for fp32/bf16/fp16 inputs),
# which differs from the division in the last bit for some inputs. The
# reference quantizes where its weights live -- on the GPU in a served
# engine -- so ``device="cuda"`` (the default) is the deployed behaviour and
# the one the library follows; ``device="cpu"`` is what the golden vectors
# record, as they were made by running the reference on the CPU. Tensor by
# tensor divisions (``w / scale[:, None]``) are IEEE on both devices.


def div_by_number(a, c: float, device: str) -> np.ndarray:
    """``tensor / python_number`` as torch computes it on ``device`` (fp32 math)."""
    a = np.asarray(a, dtype=np.float32)
    if device == "cpu":
        return (a / _F32(c)).astype(np.float32)
    if device == "cuda":
        return (a * (_F32(1.0) / _F32(c))).astype(np.float32)
    raise ValueError(f"device must be 'cpu' or 'cuda', got {device!r}")


def quantize_weight_per_channel(weight, device: str = "cuda") -> tuple[np.ndarray, np.ndarray]:
    """qtts/quant/int8.py:45-56 -- symmetric per-output-channel int8.

    fp32 throughout: scale = max(rowabsmax, 1e-12) / 127, q = clamp(round(w /
    scale), -127, 127) with round half to even (torch.round).
    """
    w = np.asarray(weight, dtype=np.float32)
    amax = np.abs(w).max(axis=1)
    scale = div_by_number(np.maximum(amax, _F32(1e-12)), 127.0, device)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def tune_quantize(weight_bf16, device: str = "cuda") -> tuple[np.ndarray, np.ndarray]:
    """examples/kernels/tune_w8_gemm.py:82-85 -- the tuning script's quantizer.

    scale = bf16(amax / 127) (no 1e-12 floor), packed = round(w / float(scale)).
    """
    w = np.asarray(weight_bf16, dtype=np.float32)
    scale = bf16_round(div_by_number(np.abs(w).max(axis=1), 127.0, device))
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def quantize_weight_fp8(weight, device: str = "cuda") -> tuple[np.ndarray, np.ndarray]:
    """qtts/quant/fp8.py:45-49 -- per-output-channel e4m3, scale = max(amax, 1e-12) / 448."""
    w = np.asarray(weight, dtype=np.float32)
    amax = np.abs(w).max(axis=1)
    scale = div_by_number(np.maximum(amax, _F32(1e-12)), 448.0, device)
    return e4m3_encode(w / scale[:, None]), scale


def quantize_act_fp8(x, dtype: str = "bf16", device: str = "cuda") -> tuple[np.ndarray, np.ndarray]:
    """qtts/quant/fp8.py:77-78 -- per-token dynamic activation quantization.

    amax in the activation dtype (exact), clamp_min(1e-6) in that dtype (the
    bound is 1e-6 rounded to it), then ``.float() / 448`` and the e4m3 cast of
    ``x.float() / scale``.
    """
    xv = np.asarray(x, dtype=np.float32)
    amax = np.abs(xv).max(axis=1)
    floor = round_to(np.array([1e-6], dtype=np.float32), dtype)[0]
    scale = div_by_number(np.maximum(amax, floor), 448.0, device)
    return e4m3_encode(xv / scale[:, None]), scale


def quantize_act_int8(x, dtype: str = "bf16", device: str = "cuda") -> tuple[np.ndarray, np.ndarray]:
    """qtts/quant/int8.py:138-140 -- Int8Method's per-token activation quantization, each
    step in the activation dtype as torch evaluates it:

    amax (exact), ``clamp_min(1e-6)`` (the bound rounded to the dtype), ``/ 127`` (a
    tensor / number: on ``device``, rounded to the dtype), ``flat / scale_x`` (tensor /
    tensor: an IEEE fp32 division rounded to the dtype), ``round()`` half to even,
    clamp to +-127. Returns (q int8 [M, K], scale fp32 [M] holding the dtype scale).
    """
    xv = np.asarray(x, dtype=np.float32)
    amax = np.abs(xv).max(axis=1)
    floor = round_to(np.array([1e-6], dtype=np.float32), dtype)[0]
    c = np.maximum(amax, floor)
    scale = round_to(div_by_number(c, 127.0, device), dtype)
    with np.errstate(invalid="ignore", divide="ignore"):
        v = np.rint(round_to((xv / scale[:, None]).astype(np.float32), dtype))
    # 0 / 0 (a zero scale from an all-zero fp16 row) stays NaN through round and
    # clamp and converts to 0 on the GPU.
    q = np.where(np.isnan(v), 0.0, np.clip(v, -127, 127)).astype(np.int8)
    return q, scale.astype(np.float32)


# ----------------------------------------------------------------------------
# GEMMs


def w8a16_reference(x, q, scale, bias=None) -> np.ndarray:
    """The fused kernel's math (qtts/quant/kernels.py:114-135) in float64.

    ``x`` holds the activation values (already representable in their dtype),
    ``q`` the int8 weight, ``scale`` the per-channel scale values (as stored,
    e.g. bf16-rounded). acc = x @ q.T; out = acc * scale (+ bias).
    """
    acc = np.asarray(x, dtype=np.float64) @ np.asarray(q, dtype=np.float64).T
    out = acc * np.asarray(scale, dtype=np.float64)[None, :]
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float64)[None, :]
    return out


def naive_dequant_linear(x_bf16, q, scale_bf16) -> np.ndarray:
    """examples/kernels/tune_w8_gemm.py:73-79 -- the reference's eager path.

    ``F.linear(x, q.to(bf16) * scale[:, None])``: the dequantized weight is
    rounded to bf16, the product accumulated in fp32 and rounded to bf16.
    """
    w = bf16_round(np.asarray(q, dtype=np.float32) * np.asarray(scale_bf16, dtype=np.float32)[:, None])
    acc = np.asarray(x_bf16, dtype=np.float32) @ w.T
    return bf16_round(acc)


def fp8_weight_only_reference(x, wq, scale_w, bias=None) -> np.ndarray:
    """fp8 weight-only (the method qtts/quant/fp8.py:92-122 leaves unimplemented), in float64:
    x times the decoded e4m3 weight, the per-channel scale after the sum, plus bias."""
    w = e4m3_decode(wq).astype(np.float64)
    out = (np.asarray(x, dtype=np.float64) @ w.T) * np.asarray(scale_w, dtype=np.float64).reshape(1, -1)
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float64)[None, :]
    return out


def fp8_scaled_mm_reference(xq, scale_x, wq, scale_w, bias=None) -> np.ndarray:
    """qtts/quant/fp8.py:79-88 -- ``_scaled_mm(q, W.t(), scale_a, scale_b) + bias`` in float64."""
    a = e4m3_decode(xq).astype(np.float64)
    b = e4m3_decode(wq).astype(np.float64)
    out = (a @ b.T) * np.asarray(scale_x, dtype=np.float64).reshape(-1, 1)
    out = out * np.asarray(scale_w, dtype=np.float64).reshape(1, -1)
    if bias is not None:
        out = out + np.asarray(bias, dtype=np.float64)[None, :]
    return out


def int8_w8a8_reference(xq, scale_x, wq, scale_w, bias=None) -> np.ndarray:
    """qtts/quant/int8.py:142-153 -- ``torch._int_mm`` then ``acc.float() * scale_x *
    int8_scale (+ bias)``: the exact integer sum converted to fp32, then the two products
    and the bias each rounded to fp32 in that order. Returns fp32 [M, N] (the caller
    rounds to the output dtype)."""
    acc = np.asarray(xq, dtype=np.int64) @ np.asarray(wq, dtype=np.int64).T
    y = acc.astype(np.float32)
    y = (y * np.asarray(scale_x, dtype=np.float32).reshape(-1, 1)).astype(np.float32)
    y = (y * np.asarray(scale_w, dtype=np.float32).reshape(1, -1)).astype(np.float32)
    if bias is not None:
        y = (y + np.asarray(bias, dtype=np.float32).reshape(1, -1)).astype(np.float32)
    return y


# ----------------------------------------------------------------------------
# Activation prologues (RMSNorm before a projection, SiLU·up between the MLP's)


def rms_norm_reference(x, weight, eps: float = 1e-6, dtype: str = "bf16") -> np.ndarray:
    """qtts/layers/norm.py:123-137 (RMSNorm, eager form): ``weight * (x * rsqrt(mean(x^2) +
    eps))``. Computed in float64, the value the reference's fp32 forms both approximate (its
    own test takes the same float64 answer, tests/test_norm.py:29-32), then rounded to the
    output dtype."""
    x64 = np.asarray(x, dtype=np.float64)
    w64 = np.asarray(weight, dtype=np.float64)
    inv = 1.0 / np.sqrt((x64 * x64).mean(axis=-1, keepdims=True) + eps)
    return round_to((w64 * (x64 * inv)).astype(np.float32), dtype)


def float_steps(a, b, dtype: str) -> np.ndarray:
    """How many representable values of ``dtype`` lie between ``a`` and ``b`` (both holding
    values of that dtype): bit patterns mapped to integers in float order, as the
    reference's norm test counts them (tests/test_norm.py:40-52)."""
    def order(v):
        v = np.asarray(v, dtype=np.float32)
        if dtype == "bf16":
            bits = (v.view(np.uint32) >> 16).astype(np.int64)
            sign, mag = bits >> 15, bits & 0x7FFF
        elif dtype == "fp16":
            bits = v.astype(np.float16).view(np.uint16).astype(np.int64)
            sign, mag = bits >> 15, bits & 0x7FFF
        else:
            bits = v.view(np.uint32).astype(np.int64)
            sign, mag = bits >> 31, bits & 0x7FFFFFFF
        return np.where(sign == 1, -mag, mag)
    return np.abs(order(a) - order(b))


def silu_mul_reference(gate, up, dtype: str = "bf16") -> np.ndarray:
    """qtts/layers/activation.py:147 -- ``F.silu(gate) * up`` on tensors of ``dtype``:
    silu in fp32 (``g / (1 + exp(-g))``) rounded to the dtype, then the product in fp32
    rounded to the dtype (torch's two elementwise kernels)."""
    g = np.asarray(gate, dtype=np.float32)
    with np.errstate(over="ignore"):
        s = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
    s = round_to(s, dtype)
    return round_to((s * np.asarray(up, dtype=np.float32)).astype(np.float32), dtype)


def rel_err(out, ref) -> float:
    """examples/kernels/tune_w8_gemm.py:121 -- max|out - ref| / max|ref|."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.abs(ref).max()
    if denom == 0:
        return float(np.abs(out - ref).max())
    return float(np.abs(out - ref).max() / denom)
