"""The reference's own talker and code predictor with the library swapped in for its kernel.

The model is the reference's ``Qwen3TTSTalker`` / ``CodePredictor``
(qtts/models/talker.py, qtts/models/code_predictor.py) built at the config-4 sizes with
random weights, quantized by the reference's ``apply_quantization`` to int8 weight-only
with every linear converted (``exclude_substrings=()``). Three arms share the same int8
buffers and differ only in the GEMM behind ``Int8WeightOnlyMethod.apply``: the library
(the one-file swap of qtts/quant/kernels.py), the reference's Triton ``w8_gemm``, and the
reference's eager dequantize-then-matmul (examples/kernels/tune_w8_gemm.py:73-79).

Checked: identical greedy codebook-0 ids on the talker decode step at batch 8 with 512
prior tokens (the north star's config-4 criterion) against the eager path and against
Triton, with the top-1/top-2 logit margin of every row printed beside the match; the
reference's CUDA graphs (qtts/compilation.py) capture and replay the library's kernels
with results equal to the same frame run eagerly.
"""

from __future__ import annotations

import pytest
import torch

from conftest import require_b200

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rf():
    require_b200()
    from baseline import ref_frame
    from baseline.install import installed

    if not installed():
        pytest.skip("reference package not installed under baseline/_ref (python -m baseline.install)")
    return ref_frame


@pytest.fixture(scope="module")
def models(rf):
    talker, predictor, report = rf.build_models(kernels="library", quant="int8_weight_only", calibrate=False)
    yield talker, predictor, report
    del talker, predictor
    torch.cuda.empty_cache()


def _logits(rf, talker, embeds, kind):
    rf.set_kernels(kind)
    try:
        return rf.talker_step_logits(talker, embeds.clone()).float()
    finally:
        rf.set_kernels("library")


def test_every_linear_converted(models):
    _, _, report = models
    assert report["talker"]["converted"] == 28 * 4 + 1 + 2  # qkv, o, gate_up, down per layer; codec head; text MLP
    assert report["talker"]["declined"] == 0
    assert report["code_predictor"]["converted"] == 5 * 4 + 15 + 1
    assert report["code_predictor"]["declined"] == 0


def _mean_abs(a, b, finite):
    return (a - b)[finite].abs().mean().item()


def test_talker_code0_matches_reference_eager_and_triton(rf, models):
    """Greedy code 0 of the 28-layer talker step equals the reference's eager path and its
    Triton path on every row. Through 28 layers the bf16 activations drift apart by far more
    than one GEMM's error, so the logits are held to a relative criterion instead of the
    single-GEMM bar: the library's mean distance from the eager path is no larger than (1.5x)
    the reference's own Triton kernel's."""
    talker, _, _ = models
    _, embeds = rf.initial_state()
    lib = _logits(rf, talker, embeds, "library")
    eager = _logits(rf, talker, embeds, "eager")
    triton = _logits(rf, talker, embeds, "triton")

    top2 = eager.topk(2, dim=-1).values
    margins = (top2[:, 0] - top2[:, 1]).tolist()
    finite = torch.isfinite(eager)
    assert torch.equal(finite, torch.isfinite(lib)) and torch.equal(finite, torch.isfinite(triton))
    d_le, d_te, d_lt = (_mean_abs(lib, eager, finite), _mean_abs(triton, eager, finite),
                        _mean_abs(lib, triton, finite))
    print(f"\ncode0 library {lib.argmax(-1).tolist()}\ncode0 eager   {eager.argmax(-1).tolist()}"
          f"\ncode0 triton  {triton.argmax(-1).tolist()}\ntop1-top2 margins (eager logits) "
          f"{[round(m, 4) for m in margins]}\nmean |library - eager| {d_le:.5f}, mean |triton - eager| "
          f"{d_te:.5f}, mean |library - triton| {d_lt:.5f}, max |logit| {eager[finite].abs().max().item():.3f}")
    assert torch.equal(lib.argmax(-1), eager.argmax(-1)), "greedy code 0 differs from the reference's eager path"
    assert torch.equal(lib.argmax(-1), triton.argmax(-1)), "greedy code 0 differs from the reference's Triton path"
    assert d_le <= 1.5 * d_te + 1e-6


def test_reference_graphs_capture_library_kernels(rf, models):
    """One frame through TalkerDecodeGraphs / CodePredictorGraphs equals the same frame run
    eagerly (talker.decode, CodePredictor.forward) with the library's kernels."""
    talker, predictor, _ = models
    rf.set_kernels("library")
    frame = rf.RefFrame(talker, predictor)
    hidden0 = frame.hidden.clone()
    codes_graph = frame.step().clone()
    hidden_graph = frame.hidden.clone()
    torch.cuda.synchronize()

    with torch.inference_mode():
        logits = talker.logits(hidden0)
        layer0 = logits.argmax(dim=-1)
        layer0_embed = talker.embed_codec(layer0.reshape(-1, 1)).squeeze(1)
        codes = predictor(layer0, layer0_embed, hidden0, do_sample=False)
        gathered = frame.residual[frame.row_index, codes[:, 1:]]
        next_embeds = layer0_embed + gathered.sum(dim=1) + talker.tts_pad_embed
        seq_lens = torch.full((frame.batch,), rf.PRIOR_TOKENS, dtype=torch.long, device=hidden0.device)
        active = torch.ones(frame.batch, dtype=torch.bool, device=hidden0.device)
        hidden = talker.decode(next_embeds, seq_lens, rf.PRIOR_TOKENS + 1, active)
    assert torch.equal(codes_graph, codes)
    assert torch.equal(hidden_graph, hidden)
    assert frame.graphs.stats()["graphs"] == 1 and frame.pgraphs.stats()["graphs"] == 1


def test_code_predictor_against_triton(rf, models):
    """The code predictor under the library against the reference's Triton kernel and eager
    path: the first codebook step's head logits (prefix of 2 positions through the 5 layers
    and lm_head[0]) no farther (1.5x) from the eager path than Triton's, code 0 equal, and the
    match rate of codes 1..15 reported (library and Triton compute the exact-int8 product with
    fp32 accumulation, so later codes can differ only where accumulation order flips a near
    tie and the walk then diverges)."""
    talker, predictor, _ = models
    hidden, _ = rf.initial_state()
    codes, first = {}, {}
    for kind in ("library", "triton", "eager"):
        rf.set_kernels(kind)
        with torch.inference_mode():
            layer0 = talker.logits(hidden).argmax(dim=-1)
            embed = talker.embed_codec(layer0.reshape(-1, 1)).squeeze(1)
            codes[kind] = predictor(layer0, embed, hidden, do_sample=False)
            proj = predictor.small_to_mtp_projection
            seq = torch.stack([proj(hidden), proj(embed)], dim=1)
            pos = torch.arange(2, device=hidden.device).expand(hidden.shape[0], 2)
            first[kind] = predictor.lm_head[0](predictor._prefix(seq, pos)[:, 1]).float()
    rf.set_kernels("library")
    match = (codes["library"][:, 1:] == codes["triton"][:, 1:]).float().mean().item()
    every = torch.ones_like(first["eager"], dtype=torch.bool)
    d_le = _mean_abs(first["library"], first["eager"], every)
    d_te = _mean_abs(first["triton"], first["eager"], every)
    print(f"\ncodes 1..15 library == triton: {match:.3f}; first head logits mean |library - eager| {d_le:.5f}, "
          f"mean |triton - eager| {d_te:.5f}")
    assert torch.equal(codes["library"][:, 0], codes["triton"][:, 0])
    assert d_le <= 1.5 * d_te + 1e-6
