"""Fused dequantize-and-matmul entry points on the sm_100a library.

Drop-in for ``qtts/quant/kernels.py``: ``kernel_available()`` and
``w8_gemm(x, weight, scale, bias=None)`` keep their names, argument meaning
and error behaviour (kernels.py:84-86, 138-177), but the work is done by the
hand-written CUDA kernels behind the C ABI (``include/qtts_b200.h``) instead of
Triton. Every function launches on ``torch.cuda.current_stream()`` and
allocates only its output (from torch's caching allocator), so all of them can
be captured in a CUDA graph.

There is no CPU path. CPU tensors, or a machine without the library or a
compute-capability 10.x GPU, raise ``RuntimeError``.
"""

from __future__ import annotations

import torch

from .. import _native as nat

#: Launch with programmatic dependent launch unless told otherwise. Safe for
#: every kernel of this library: weights are never written by the kernel that
#: immediately precedes a GEMM, and everything else is read after the wait.
USE_PDL = True


def kernel_available() -> tuple[bool, str]:
    """(available, reason) -- the library loaded and an sm_100 GPU is present."""
    return nat.available()


def _flags() -> int:
    return nat.FLAG_PDL if USE_PDL else 0


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise RuntimeError(f"qtts_b200 kernels run on CUDA tensors only, got a tensor on {t.device}")
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError(f"tensors on different devices: {device} and {t.device}")
    assert device is not None
    return device


def _rows_view(x: torch.Tensor, k: int) -> torch.Tensor:
    """[..., K] -> a 2-D [rows, K] view with unit stride along K (copying only if needed)."""
    a = x.reshape(-1, k) if x.dim() != 2 else x
    if a.stride(-1) != 1 or (a.shape[0] > 1 and a.stride(0) < k):
        a = a.contiguous()
    return a


def w8_gemm(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    variant: int = nat.VARIANT_AUTO,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``x @ (weight * scale).T + bias``, dequantizing ``weight`` in registers.

    ``x`` is ``[..., K]`` (bf16, fp16 or fp32), ``weight`` is ``[N, K]`` int8 and
    ``scale`` is ``[N]`` (bf16, fp16 or fp32): one per output channel, applied
    once after the fp32 K loop. The result has ``x``'s dtype and shape
    ``[..., N]``. ``variant`` selects a kernel (see ``include/qtts_b200.h``);
    the default lets the library choose.
    """
    if weight.dim() != 2 or weight.dtype != torch.int8:
        raise ValueError(f"weight must be a 2-D int8 tensor, got {tuple(weight.shape)} {weight.dtype}")
    return _weight_only_gemm(x, weight, scale, bias, variant, out, "qtts_w8a16_gemm")


def fp8w_gemm(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    variant: int = nat.VARIANT_AUTO,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """fp8 weight-only: ``x @ (e4m3(weight) * scale).T + bias``, the W8A16 contract with an
    e4m3 ``[N, K]`` weight (``torch.float8_e4m3fn``, row-major) converted in registers."""
    if weight.dim() != 2 or weight.dtype != torch.float8_e4m3fn:
        raise ValueError(f"weight must be a 2-D float8_e4m3fn tensor, got {tuple(weight.shape)} {weight.dtype}")
    return _weight_only_gemm(x, weight, scale, bias, variant, out, "qtts_fp8w_gemm")


def _weight_only_gemm(x, weight, scale, bias, variant, out, entry: str) -> torch.Tensor:
    ok, reason = nat.available()
    if not ok:
        raise RuntimeError(reason)
    shape = x.shape
    k = shape[-1]
    n = weight.shape[0]
    if weight.shape[1] != k:
        raise ValueError(f"weight is [{n}, {weight.shape[1]}] but x has K={k}")
    if scale.numel() != n:
        raise ValueError(f"scale has {scale.numel()} elements, expected {n}")
    device = _require_cuda(x, weight, scale, bias)
    a = _rows_view(x, k)
    rows = a.shape[0]
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    scale = scale.reshape(-1)
    if scale.stride(0) != 1:
        scale = scale.contiguous()
    if bias is not None:
        bias = bias.reshape(-1)
        if bias.dtype != x.dtype or bias.stride(0) != 1:
            bias = bias.to(x.dtype).contiguous()
    if out is None:
        out = torch.empty((rows, n), device=device, dtype=x.dtype)
    elif out.shape != (rows, n) or out.dtype != x.dtype or out.stride(1) != 1:
        raise ValueError(f"out must be [{rows}, {n}] {x.dtype} with unit column stride")
    code = getattr(nat.lib(), entry)(
        a.data_ptr(), a.stride(0) if rows > 1 else k, nat.dtype_code(a.dtype),
        weight.data_ptr(), weight.stride(0),
        scale.data_ptr(), nat.dtype_code(scale.dtype),
        bias.data_ptr() if bias is not None else None,
        out.data_ptr(), out.stride(0) if rows > 1 else n,
        rows, n, k, variant, _flags(), nat.stream_ptr(device),
    )
    nat.check(code, entry)
    return out.reshape(*shape[:-1], n)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, *,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over the last dimension (qtts/layers/norm.py:49-76, 102-137):
    ``cast(weight * (x * (1 / sqrt(mean(x^2) + eps))))`` in fp32, the sum of
    squares in the library's fixed order. ``weight`` is ``[W]``; bf16, fp16 or
    fp32 like ``x``. ``out`` may be ``x`` itself."""
    ok, reason = nat.available()
    if not ok:
        raise RuntimeError(reason)
    width = x.shape[-1]
    if weight.numel() != width:
        raise ValueError(f"weight has {weight.numel()} elements, expected {width}")
    device = _require_cuda(x, weight)
    a = _rows_view(x, width)
    rows = a.shape[0]
    weight = weight.reshape(-1)
    if weight.dtype != x.dtype or weight.stride(0) != 1:
        weight = weight.to(x.dtype).contiguous()
    if out is None:
        out = torch.empty((rows, width), device=device, dtype=x.dtype)
    else:
        out = _rows_view(out, width)
        if out.shape != (rows, width) or out.dtype != x.dtype or out.stride(1) != 1:
            raise ValueError(f"out must be [{rows}, {width}] {x.dtype} with unit column stride")
    code = nat.lib().qtts_rms_norm(
        a.data_ptr(), a.stride(0) if rows > 1 else width, weight.data_ptr(), out.data_ptr(),
        out.stride(0) if rows > 1 else width, nat.dtype_code(x.dtype), rows, width, float(eps), _flags(),
        nat.stream_ptr(device))
    nat.check(code, "qtts_rms_norm")
    return out.reshape(*x.shape)


def silu_mul(gate_up: torch.Tensor, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """``F.silu(gate) * up`` of ``gate_up = [gate | up]`` (``[..., 2W]`` -> ``[..., W]``;
    qtts/layers/activation.py:143-147), bit for bit torch's two CUDA kernels."""
    ok, reason = nat.available()
    if not ok:
        raise RuntimeError(reason)
    two_w = gate_up.shape[-1]
    if two_w % 2:
        raise ValueError(f"gate_up last dimension {two_w} is odd")
    width = two_w // 2
    device = _require_cuda(gate_up)
    a = _rows_view(gate_up, two_w)
    rows = a.shape[0]
    if out is None:
        out = torch.empty((rows, width), device=device, dtype=gate_up.dtype)
    elif out.shape != (rows, width) or out.dtype != gate_up.dtype or out.stride(1) != 1:
        raise ValueError(f"out must be [{rows}, {width}] {gate_up.dtype} with unit column stride")
    code = nat.lib().qtts_silu_mul(
        a.data_ptr(), a.stride(0) if rows > 1 else two_w, out.data_ptr(), out.stride(0) if rows > 1 else width,
        nat.dtype_code(gate_up.dtype), rows, width, _flags(), nat.stream_ptr(device))
    nat.check(code, "qtts_silu_mul")
    return out.reshape(*gate_up.shape[:-1], width)


_HEAD_STATE: dict[int, torch.Tensor] = {}


def _head_state(device: torch.device) -> torch.Tensor:
    """The zeroed uint64 state words of ``qtts_w8a16_head_argmax`` on ``device`` (17: up to 16
    rows + a CTA counter). Every call leaves them zero, so calls ordered on one stream share
    them; allocated on the first call (make one before capturing a CUDA graph)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _HEAD_STATE.get(idx)
    if st is None:
        st = torch.zeros(17, dtype=torch.int64, device=device)
        _HEAD_STATE[idx] = st
    return st


def w8_head_argmax(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    *,
    norm_weight: torch.Tensor | None = None,
    eps: float = 1e-6,
    logit_bias: torch.Tensor | None = None,
    embed: torch.Tensor | None = None,
    codes: torch.Tensor | None = None,
    embed_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """The end of a greedy decode step in one launch (``qtts_w8a16_head_argmax``):
    ``codes = (rms_norm(x) @ (weight * scale).T (+ logit_bias)).argmax(-1)`` with the logits
    rounded to x's dtype as the head's output is, and ``embed[codes]`` gathered when ``embed``
    is given (the next step's input row). x ``[M, K]`` (M <= 16, K % 128 == 0, K <= 2048),
    weight ``[N, K]`` int8, scale ``[N]``, logit_bias ``[N]`` fp32 (0 / -inf mask), embed
    ``[vocab, E]`` in x's dtype. Returns ``(codes [M] int64, embed rows [M, E] or None)``."""
    ok, reason = nat.available()
    if not ok:
        raise RuntimeError(reason)
    if x.dim() != 2 or weight.dim() != 2 or weight.shape[1] != x.shape[1]:
        raise ValueError(f"x {tuple(x.shape)} and weight {tuple(weight.shape)} do not agree")
    m, k = x.shape
    n = weight.shape[0]
    device = _require_cuda(x, weight, scale, norm_weight, logit_bias, embed)
    if x.stride(1) != 1:
        x = x.contiguous()
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    scale = scale.reshape(-1).contiguous()
    if norm_weight is not None:
        norm_weight = norm_weight.reshape(-1).to(x.dtype).contiguous()
    if logit_bias is not None:
        logit_bias = logit_bias.reshape(-1).to(torch.float32).contiguous()
    if codes is None:
        codes = torch.empty(m, dtype=torch.int64, device=device)
    e = vocab = 0
    if embed is not None:
        if embed.dim() != 2 or embed.dtype != x.dtype or embed.stride(1) != 1:
            raise ValueError("embed must be a [vocab, E] table of x's dtype with unit column stride")
        vocab, e = embed.shape
        if embed_out is None:
            embed_out = torch.empty((m, e), dtype=x.dtype, device=device)
    state = _head_state(device)
    code = nat.lib().qtts_w8a16_head_argmax(
        x.data_ptr(), x.stride(0) if m > 1 else k, nat.dtype_code(x.dtype),
        norm_weight.data_ptr() if norm_weight is not None else None, float(eps),
        weight.data_ptr(), weight.stride(0) if n > 1 else k, scale.data_ptr(), nat.dtype_code(scale.dtype),
        logit_bias.data_ptr() if logit_bias is not None else None, codes.data_ptr(),
        embed.data_ptr() if embed is not None else None, embed.stride(0) if embed is not None else 0, vocab,
        embed_out.data_ptr() if embed is not None else None, embed_out.stride(0) if embed is not None else 0, e,
        state.data_ptr(), m, n, k, _flags(), nat.stream_ptr(device))
    nat.check(code, "qtts_w8a16_head_argmax")
    return codes, (embed_out if embed is not None else None)


def prologue_fused(m: int, n: int, k: int, prologue: int, variant: int = nat.VARIANT_AUTO) -> bool:
    """Whether ``w8_gemm_rmsnorm`` / ``w8_gemm_silu_mul`` of this shape runs as one launch."""
    return bool(nat.lib().qtts_w8a16_gemm_prologue_fused(m, n, k, prologue, variant))


def _prologue_gemm(x, prologue, norm_weight, eps, weight, scale, bias, variant) -> torch.Tensor:
    ok, reason = nat.available()
    if not ok:
        raise RuntimeError(reason)
    if weight.dim() != 2 or weight.dtype != torch.int8:
        raise ValueError(f"weight must be a 2-D int8 tensor, got {tuple(weight.shape)} {weight.dtype}")
    n, k = weight.shape
    width = 2 * k if prologue == nat.PROLOGUE_SILU_MUL else k
    if x.shape[-1] != width:
        raise ValueError(f"x has last dimension {x.shape[-1]}, expected {width} for weight [{n}, {k}]")
    if scale.numel() != n:
        raise ValueError(f"scale has {scale.numel()} elements, expected {n}")
    device = _require_cuda(x, weight, scale, bias, norm_weight)
    a = _rows_view(x, width)
    rows = a.shape[0]
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    scale = scale.reshape(-1)
    if scale.stride(0) != 1:
        scale = scale.contiguous()
    if bias is not None:
        bias = bias.reshape(-1)
        if bias.dtype != x.dtype or bias.stride(0) != 1:
            bias = bias.to(x.dtype).contiguous()
    if norm_weight is not None:
        norm_weight = norm_weight.reshape(-1)
        if norm_weight.numel() != k:
            raise ValueError(f"norm weight has {norm_weight.numel()} elements, expected {k}")
        if norm_weight.dtype != x.dtype or norm_weight.stride(0) != 1:
            norm_weight = norm_weight.to(x.dtype).contiguous()
    out = torch.empty((rows, n), device=device, dtype=x.dtype)
    workspace = None
    if rows > 0 and not prologue_fused(rows, n, k, prologue, variant):
        workspace = torch.empty((rows, k), device=device, dtype=x.dtype)
    code = nat.lib().qtts_w8a16_gemm_prologue(
        a.data_ptr(), a.stride(0) if rows > 1 else width, nat.dtype_code(a.dtype), prologue,
        norm_weight.data_ptr() if norm_weight is not None else None, float(eps),
        weight.data_ptr(), weight.stride(0), scale.data_ptr(), nat.dtype_code(scale.dtype),
        bias.data_ptr() if bias is not None else None, out.data_ptr(), n, rows, n, k,
        workspace.data_ptr() if workspace is not None else None, variant, _flags(), nat.stream_ptr(device))
    nat.check(code, "qtts_w8a16_gemm_prologue")
    return out.reshape(*x.shape[:-1], n)


def w8_gemm_rmsnorm(x: torch.Tensor, norm_weight: torch.Tensor, eps: float, weight: torch.Tensor,
                    scale: torch.Tensor, bias: torch.Tensor | None = None, *,
                    variant: int = nat.VARIANT_AUTO) -> torch.Tensor:
    """``w8_gemm(rms_norm(x, norm_weight, eps), weight, scale, bias)`` -- one launch when the
    chosen kernel stages activations itself (one of the two streaming kernels, M <= 16), else
    the norm kernel chained ahead (``prologue_fused`` tells which)."""
    return _prologue_gemm(x, nat.PROLOGUE_RMSNORM, norm_weight, eps, weight, scale, bias, variant)


def w8_gemm_silu_mul(gate_up: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor,
                     bias: torch.Tensor | None = None, *, variant: int = nat.VARIANT_AUTO) -> torch.Tensor:
    """``w8_gemm(silu_mul(gate_up), weight, scale, bias)`` (the down projection of a gated MLP)."""
    return _prologue_gemm(gate_up, nat.PROLOGUE_SILU_MUL, None, 0.0, weight, scale, bias, variant)


def w8_gemm_allgather(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor | None,
    *,
    peer_out: torch.Tensor,
    ldo: int,
    col_offset: int,
    peer_signal: torch.Tensor,
    sync: torch.Tensor,
    rank: int,
    world: int,
    variant: int = nat.VARIANT_AUTO,
) -> None:
    """This rank's block of an N-sharded W8A16 GEMM, stored by the kernel into every
    rank's gathered output (``qtts_w8a16_gemm_allgather``).

    ``peer_out`` / ``peer_signal``: int64 CUDA tensors of ``world`` device addresses
    (each rank's gathered buffer and signal pad, this rank's own at ``rank``);
    ``sync``: this rank's int32 [2] CUDA tensor. The gathered buffers hold rows of
    ``ldo`` elements of x's dtype; this rank's block lands at columns
    ``[col_offset, col_offset + N)``.
    """
    ok, reason = nat.available()
    if not ok:
        raise RuntimeError(reason)
    k = x.shape[-1]
    n = weight.shape[0]
    if x.dim() != 2 or weight.dim() != 2 or weight.shape[1] != k or scale.numel() != n:
        raise ValueError(f"x {tuple(x.shape)}, weight {tuple(weight.shape)}, scale {scale.numel()} do not agree")
    for name, t, dt, numel in (("peer_out", peer_out, torch.int64, world), ("peer_signal", peer_signal, torch.int64,
                                                                             world), ("sync", sync, torch.int32, 2)):
        if t.dtype != dt or t.numel() != numel or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dt} tensor of {numel} elements")
    device = _require_cuda(x, weight, scale, bias, peer_out, peer_signal, sync)
    if x.stride(1) != 1:
        x = x.contiguous()
    if weight.stride(1) != 1:
        weight = weight.contiguous()
    scale = scale.reshape(-1).contiguous()
    if bias is not None:
        bias = bias.reshape(-1).to(x.dtype).contiguous()
    rows = x.shape[0]
    code = nat.lib().qtts_w8a16_gemm_allgather(
        x.data_ptr(), x.stride(0) if rows > 1 else k, nat.dtype_code(x.dtype),
        weight.data_ptr(), weight.stride(0),
        scale.data_ptr(), nat.dtype_code(scale.dtype),
        bias.data_ptr() if bias is not None else None,
        peer_out.data_ptr(), ldo, col_offset, peer_signal.data_ptr(), sync.data_ptr(),
        rank, world, rows, n, k, variant, _flags(), nat.stream_ptr(device),
    )
    nat.check(code, "qtts_w8a16_gemm_allgather")


def w8_grouped_gemm(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    variant: int = nat.VARIANT_AUTO,
) -> torch.Tensor:
    """G independent W8A16 problems of one shape in one launch.

    ``x`` is ``[G, M, K]``, ``weight`` the stacked ``[G*N, K]`` int8 matrix,
    ``scale`` ``[G*N]``; returns ``[G, M, N]``.
    """
    ok, reason = nat.available()
    if not ok:
        raise RuntimeError(reason)
    if x.dim() != 3:
        raise ValueError("x must be [G, M, K]")
    g, m, k = x.shape
    if weight.shape[0] % g != 0 or weight.shape[1] != k:
        raise ValueError(f"weight {tuple(weight.shape)} is not [G*N, {k}] for G={g}")
    n = weight.shape[0] // g
    device = _require_cuda(x, weight, scale, bias)
    if x.stride(2) != 1:
        x = x.contiguous()
    if bias is not None and bias.dtype != x.dtype:
        bias = bias.to(x.dtype)
    out = torch.empty((g, m, n), device=device, dtype=x.dtype)
    code = nat.lib().qtts_w8a16_grouped_gemm(
        x.data_ptr(), x.stride(0), x.stride(1) if m > 1 else k, nat.dtype_code(x.dtype),
        weight.data_ptr(), weight.stride(0),
        scale.data_ptr(), nat.dtype_code(scale.dtype),
        bias.data_ptr() if bias is not None else None,
        out.data_ptr(), out.stride(0), n,
        g, m, n, k, None, variant, _flags(), nat.stream_ptr(device),
    )
    nat.check(code, "qtts_w8a16_grouped_gemm")
    return out


def w8_indexed_gemm(
    x: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    index: torch.Tensor,
    groups: int,
    bias: torch.Tensor | None = None,
    *,
    out: torch.Tensor | None = None,
    variant: int = nat.VARIANT_AUTO,
) -> torch.Tensor:
    """One group of a stacked ``[groups*N, K]`` weight, chosen by a device tensor.

    ``index`` is a one-element int64 CUDA tensor read by the kernel at run
    time, so a captured graph can pick a different codebook head per replay.
    ``x`` is ``[M, K]``; returns ``[M, N]``.
    """
    ok, reason = nat.available()
    if not ok:
        raise RuntimeError(reason)
    k = x.shape[-1]
    a = _rows_view(x, k)
    m = a.shape[0]
    n = weight.shape[0] // groups
    device = _require_cuda(a, weight, scale, bias, index)
    if index.dtype != torch.int64 or index.numel() != 1:
        raise ValueError("index must be a one-element int64 tensor")
    if bias is not None and bias.dtype != x.dtype:
        bias = bias.to(x.dtype)
    if out is None:
        out = torch.empty((m, n), device=device, dtype=x.dtype)
    code = nat.lib().qtts_w8a16_grouped_gemm(
        a.data_ptr(), 0, a.stride(0) if m > 1 else k, nat.dtype_code(a.dtype),
        weight.data_ptr(), weight.stride(0),
        scale.data_ptr(), nat.dtype_code(scale.dtype),
        bias.data_ptr() if bias is not None else None,
        out.data_ptr(), 0, out.stride(0) if m > 1 else n,
        groups, m, n, k, index.data_ptr(), variant, _flags(), nat.stream_ptr(device),
    )
    nat.check(code, "qtts_w8a16_grouped_gemm (indexed)")
    return out.reshape(*x.shape[:-1], n)


def quantize_int8_rows(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel int8 on the GPU; bit-exact with quantize_weight_per_channel."""
    device = _require_cuda(weight)
    w = weight.detach()
    if w.stride(-1) != 1:
        w = w.contiguous()
    n, k = w.shape
    q = torch.empty((n, k), device=device, dtype=torch.int8)
    s = torch.empty((n,), device=device, dtype=torch.float32)
    code = nat.lib().qtts_quantize_int8_rows(
        w.data_ptr(), w.stride(0), nat.dtype_code(w.dtype), q.data_ptr(), s.data_ptr(), n, k,
        nat.stream_ptr(device),
    )
    nat.check(code, "qtts_quantize_int8_rows")
    return q, s


def quantize_fp8_rows(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel e4m3 on the GPU; bit-exact with quantize_weight_fp8."""
    device = _require_cuda(weight)
    w = weight.detach()
    if w.stride(-1) != 1:
        w = w.contiguous()
    n, k = w.shape
    q = torch.empty((n, k), device=device, dtype=torch.float8_e4m3fn)
    s = torch.empty((n,), device=device, dtype=torch.float32)
    code = nat.lib().qtts_quantize_fp8_rows(
        w.data_ptr(), w.stride(0), nat.dtype_code(w.dtype), q.data_ptr(), s.data_ptr(), n, k,
        nat.stream_ptr(device),
    )
    nat.check(code, "qtts_quantize_fp8_rows")
    return q, s


def fp8_quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token e4m3 activation quantization: returns (q [M, K], scale_x [M, 1] fp32)."""
    device = _require_cuda(x)
    k = x.shape[-1]
    a = _rows_view(x, k)
    m = a.shape[0]
    q = torch.empty((m, k), device=device, dtype=torch.float8_e4m3fn)
    s = torch.empty((m, 1), device=device, dtype=torch.float32)
    code = nat.lib().qtts_fp8_quant_rows(
        a.data_ptr(), a.stride(0) if m > 1 else k, nat.dtype_code(a.dtype), q.data_ptr(), s.data_ptr(), m, k,
        _flags(), nat.stream_ptr(device),
    )
    nat.check(code, "qtts_fp8_quant_rows")
    return q, s


def fp8_scaled_mm(
    xq: torch.Tensor,
    scale_x: torch.Tensor,
    wq: torch.Tensor,
    scale_w: torch.Tensor,
    bias: torch.Tensor | None,
    out_dtype: torch.dtype,
    *,
    variant: int = nat.VARIANT_AUTO,
) -> torch.Tensor:
    """``(xq @ wq.T) * scale_x * scale_w + bias`` with e4m3 operands.

    ``xq`` [M, K] e4m3, ``wq`` [N, K] e4m3 (row-major; pass ``fp8_weight.t()``
    of the reference's column-major view), scales fp32 ``[M]``/``[N]``.
    """
    device = _require_cuda(xq, scale_x, wq, scale_w, bias)
    m, k = xq.shape
    n = wq.shape[0]
    if wq.shape[1] != k or wq.stride(1) != 1 or xq.stride(1) != 1:
        raise ValueError("xq and wq must be row-major [M, K] and [N, K]")
    if bias is not None and bias.dtype != out_dtype:
        bias = bias.to(out_dtype)
    out = torch.empty((m, n), device=device, dtype=out_dtype)
    code = nat.lib().qtts_fp8_gemm(
        xq.data_ptr(), xq.stride(0) if m > 1 else k, scale_x.data_ptr(),
        wq.data_ptr(), wq.stride(0), scale_w.data_ptr(),
        bias.data_ptr() if bias is not None else None,
        out.data_ptr(), n, nat.dtype_code(out_dtype), m, n, k, variant, _flags(), nat.stream_ptr(device),
    )
    nat.check(code, "qtts_fp8_gemm")
    return out


def int8_quant_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token int8 activation quantization of Int8Method (qtts/quant/int8.py:138-140):
    returns (q [M, K] int8, scale_x [M, 1] fp32 holding the activation-dtype scale)."""
    device = _require_cuda(x)
    k = x.shape[-1]
    a = _rows_view(x, k)
    m = a.shape[0]
    q = torch.empty((m, k), device=device, dtype=torch.int8)
    s = torch.empty((m, 1), device=device, dtype=torch.float32)
    code = nat.lib().qtts_int8_quant_rows(
        a.data_ptr(), a.stride(0) if m > 1 else k, nat.dtype_code(a.dtype), q.data_ptr(), s.data_ptr(), m, k,
        _flags(), nat.stream_ptr(device),
    )
    nat.check(code, "qtts_int8_quant_rows")
    return q, s


def i8_scaled_mm(
    xq: torch.Tensor,
    scale_x: torch.Tensor,
    wq: torch.Tensor,
    scale_w: torch.Tensor,
    bias: torch.Tensor | None,
    out_dtype: torch.dtype,
    *,
    variant: int = nat.VARIANT_AUTO,
) -> torch.Tensor:
    """``((float(xq @ wq.T) * scale_x) * scale_w) + bias`` with int8 operands and an exact
    int32 sum (torch._int_mm and the scaling of Int8Method.apply, qtts/quant/int8.py:142-153).

    ``xq`` [M, K] int8, ``wq`` [N, K] int8 row-major (``int8_weight.t()`` of the
    reference's [K, N] layout), scales fp32 ``[M]``/``[N]``.
    """
    device = _require_cuda(xq, scale_x, wq, scale_w, bias)
    if xq.dtype != torch.int8 or wq.dtype != torch.int8:
        raise ValueError("xq and wq must be int8")
    m, k = xq.shape
    n = wq.shape[0]
    if wq.shape[1] != k or wq.stride(1) != 1 or xq.stride(1) != 1:
        raise ValueError("xq and wq must be row-major [M, K] and [N, K]")
    scale_x = scale_x.reshape(-1).to(torch.float32).contiguous()
    scale_w = scale_w.reshape(-1).to(torch.float32).contiguous()
    if bias is not None:
        bias = bias.reshape(-1).to(out_dtype).contiguous()
    out = torch.empty((m, n), device=device, dtype=out_dtype)
    code = nat.lib().qtts_i8_gemm(
        xq.data_ptr(), xq.stride(0) if m > 1 else k, scale_x.data_ptr(),
        wq.data_ptr(), wq.stride(0), scale_w.data_ptr(),
        bias.data_ptr() if bias is not None else None,
        out.data_ptr(), n, nat.dtype_code(out_dtype), m, n, k, variant, _flags(), nat.stream_ptr(device),
    )
    nat.check(code, "qtts_i8_gemm")
    return out
