"""The fused codebook head (qtts_w8a16_head_argmax) against the oracle and the unfused path.

One launch computes RMSNorm -> the int8 head -> logits rounded to the activation
dtype (+ an optional fp32 mask) -> the greedy code -> the embedding row of that code.
Checked on the code predictor's head (1024 -> 2048, batch 8) and the talker's masked
codec head (2048 -> 3072): every code is a maximum of the exact (float64) logits of the
same normalized activations up to the rounding of the head's output (a code off the
exact argmax must be within two bf16 steps of the maximum, and such rows are rare), it
equals the argmax of the library's unfused head wherever that head's top-2 margin exceeds
two bf16 steps, masked columns are never chosen, the embedding rows are the table rows of
the codes bit for bit, and repeated calls and CUDA-graph replays (the state array resets
itself) stay correct.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from conftest import require_b200
from qtts_b200 import _native as nat
from qtts_b200.quant import kernels as qk

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    require_b200()
    nat.device_status(reset=True)
    yield
    torch.cuda.synchronize()
    assert nat.device_status() == 0


def _case(m, n, k, vocab_e, e, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    q, s = oracle.quantize_weight_per_channel(w.numpy())
    x = (torch.randn(m, k, generator=g) * 3).to(dtype)
    nw = (1 + 0.1 * torch.randn(k, generator=g)).to(dtype)
    table = (torch.randn(vocab_e, e, generator=g) * 0.02).to(dtype)
    return (x.cuda(), torch.from_numpy(q).cuda(), torch.from_numpy(s).to(dtype).cuda(), nw.cuda(), table.cuda())


def _check(codes, emb_out, x, q, s, nw, table, bias=None, what=""):
    y = qk.rms_norm(x, nw, 1e-6) if nw is not None else x
    exact = y.double() @ (q.double() * s.double()[:, None]).T
    if bias is not None:
        exact = exact + bias.double()
    mx = exact.max(dim=-1).values
    picked = exact.gather(1, codes[:, None].long())[:, 0]
    step = mx.abs() * 2.0 ** -7  # one bf16 step at the maximum
    assert bool((picked >= mx - 2 * step - 1e-6).all()), f"{what}: a code is not a maximum"
    exact_codes = exact.argmax(dim=-1)
    off = int((codes != exact_codes).sum())
    assert off <= max(1, codes.numel() // 8), f"{what}: {off} rows off the exact argmax"
    # The library's unfused head: same norm, the W8A16 GEMM, rounded logits, torch's argmax.
    logits = qk.w8_gemm(y, q, s).float()
    if bias is not None:
        logits = logits + bias
    top2 = logits.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > 2 * top2[:, 0].abs() * 2.0 ** -7
    assert torch.equal(codes[clear], logits.argmax(dim=-1)[clear]), f"{what}: differs from the unfused head"
    if table is not None:
        assert torch.equal(emb_out, table[codes]), f"{what}: embedding rows"
    return off


@pytest.mark.parametrize("m", [1, 3, 8, 16])
def test_predictor_head(m):
    x, q, s, nw, table = _case(m, 2048, 1024, 2048, 1024, seed=500 + m)
    codes, emb = qk.w8_head_argmax(x, q, s, norm_weight=nw, embed=table)
    torch.cuda.synchronize()
    assert codes.shape == (m,) and codes.dtype == torch.int64 and emb.shape == (m, 1024)
    _check(codes, emb, x, q, s, nw, table, what=f"predictor M={m}")


def test_talker_codec_head_masked():
    m, n, k = 8, 3072, 2048
    x, q, s, nw, table = _case(m, n, k, 3072, 2048, seed=510)
    bias = torch.full((n,), float("-inf"), device="cuda")
    bias[1:2048] = 0.0
    bias[2150] = 0.0
    codes, emb = qk.w8_head_argmax(x, q, s, norm_weight=nw, logit_bias=bias, embed=table)
    torch.cuda.synchronize()
    allowed = ((codes >= 1) & (codes < 2048)) | (codes == 2150)
    assert bool(allowed.all())
    _check(codes, emb, x, q, s, nw, table, bias=bias, what="codec head")


def test_no_norm_no_embed_fp16():
    x, q, s, _, _ = _case(4, 1024, 2048, 8, 8, seed=520, dtype=torch.float16)
    codes, emb = qk.w8_head_argmax(x, q, s)
    torch.cuda.synchronize()
    assert emb is None
    _check(codes, None, x, q, s, None, None, what="no norm, fp16")


def test_repeated_calls_and_graph_replays():
    x, q, s, nw, table = _case(8, 2048, 1024, 2048, 1024, seed=530)
    for call in range(3):
        xc = (torch.randn(8, 1024, generator=torch.Generator().manual_seed(531 + call)) * 3).to(torch.bfloat16).cuda()
        codes, emb = qk.w8_head_argmax(xc, q, s, norm_weight=nw, embed=table)
        torch.cuda.synchronize()
        _check(codes, emb, xc, q, s, nw, table, what=f"call {call}")
    xs = x.clone()
    codes = torch.empty(8, dtype=torch.int64, device="cuda")
    emb = torch.empty(8, 1024, dtype=torch.bfloat16, device="cuda")
    qk.w8_head_argmax(xs, q, s, norm_weight=nw, embed=table, codes=codes, embed_out=emb)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        qk.w8_head_argmax(xs, q, s, norm_weight=nw, embed=table, codes=codes, embed_out=emb)
    for r in range(3):
        xn = (torch.randn(8, 1024, generator=torch.Generator().manual_seed(540 + r)) * 3).to(torch.bfloat16).cuda()
        xs.copy_(xn)
        graph.replay()
        torch.cuda.synchronize()
        _check(codes, emb, xn, q, s, nw, table, what=f"replay {r}")


def test_rejects_what_it_cannot_take():
    x, q, s, nw, table = _case(8, 256, 1024, 16, 1024, seed=550)
    with pytest.raises(RuntimeError):
        qk.w8_head_argmax(torch.zeros(17, 1024, dtype=torch.bfloat16, device="cuda"), q, s)  # M > 16
    with pytest.raises(RuntimeError):
        qk.w8_head_argmax(x[:, :1000].contiguous(), q[:, :1000].contiguous(), s)  # K % 128
    torch.cuda.synchronize()
    assert nat.device_status() == 0
    # a code beyond the embedding table is refused on the device: zeros and QTTS_ERR_SHAPE
    try:
        codes, emb = qk.w8_head_argmax(x, q, s, embed=table[:1].contiguous())
        torch.cuda.synchronize()
        if bool((codes >= 1).any()):
            assert nat.device_status() == 2  # QTTS_ERR_SHAPE
            assert not emb[codes >= 1].any()
    finally:
        nat.device_status(reset=True)
