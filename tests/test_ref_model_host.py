"""Host-side checks of the comparison harness over the reference's own model (baseline/ref_frame.py).

On the CPU the reference's model runs with its eager dequantize-then-matmul GEMM
(the Triton kernel and the library need a GPU): a two-layer talker and a one-layer
code predictor are built through the reference's ``apply_quantization`` exactly as
the config-4 benchmark builds the full model, and one talker step yields masked
logits and greedy ids. ``set_kernels`` rebinds the GEMM the reference's
``Int8WeightOnlyMethod`` calls.
"""

from __future__ import annotations

import pytest
import torch


@pytest.fixture(scope="module")
def rf():
    from baseline import ref_frame
    from baseline.install import installed

    if not installed():
        pytest.skip("reference package not installed under baseline/_ref (python -m baseline.install)")
    return ref_frame


def test_reference_model_builds_and_steps_on_cpu(rf):
    talker, predictor, report = rf.build_models(device="cpu", kernels="eager", talker_layers=2, predictor_layers=1)
    assert report["talker"]["converted"] == 2 * 4 + 3 and report["talker"]["declined"] == 0
    assert report["code_predictor"]["converted"] == 4 + 15 + 1
    assert talker.layers[0].self_attn.qkv_proj.int8_weight.dtype == torch.int8
    _, embeds = rf.initial_state(device="cpu")
    logits = rf.talker_step_logits(talker, embeds)
    assert logits.shape == (rf.BATCH, rf.CODEC_VOCAB) and logits.dtype == torch.float32
    ids = logits.argmax(-1)
    allowed = ((ids >= 1) & (ids < rf.CODE_VOCAB)) | (ids == rf.CODEC_EOS)
    assert bool(allowed.all())
    # Masked columns are -inf, everything else finite.
    assert torch.isinf(logits[:, 0]).all() and torch.isfinite(logits[:, 1:rf.CODE_VOCAB]).all()


def test_set_kernels_rebinds_the_reference_gemm(rf):
    ref = rf.qtts()
    rf.set_kernels("eager")
    assert ref.quant.int8.w8_gemm is rf.eager_w8_gemm
    rf.set_kernels("triton")
    assert ref.quant.int8.w8_gemm is ref.quant.kernels.w8_gemm
    with pytest.raises(ValueError):
        rf.set_kernels("cublas")
    rf.set_kernels("eager")


def test_eager_gemm_is_the_reference_expression(rf):
    g = torch.Generator().manual_seed(5)
    q = torch.randint(-127, 128, (64, 32), generator=g, dtype=torch.int8)
    s = (torch.rand(64, generator=g) * 0.01).to(torch.bfloat16)
    x = torch.randn(3, 32, generator=g).to(torch.bfloat16)
    want = torch.nn.functional.linear(x, q.to(torch.bfloat16) * s[:, None])
    assert torch.equal(rf.eager_w8_gemm(x, q, s), want)
