"""The reference's own talker + code predictor, run on the GPU as its engine runs them.

This builds the config-4 workload out of the reference's classes, unmodified:
``Qwen3TTSTalker`` (qtts/models/talker.py:142-356) and ``CodePredictor``
(qtts/models/code_predictor.py:133-243), quantized by the reference's
``apply_quantization`` (qtts/quant/base.py:155-183) and replayed through its
``TalkerDecodeGraphs`` / ``CodePredictorGraphs`` (qtts/compilation.py:60-273).
One frame follows ``TalkerRunner.decode_step`` (qtts/engine/talker_runner.py:180-224)
for greedy decoding with every row active: masked codec-head logits, argmax,
the code-predictor graph, the summed next-step embedding, the talker graph.

The int8 kernel under ``Int8WeightOnlyMethod`` is chosen with
:func:`set_kernels`:

* ``"triton"`` -- the reference's own ``w8_gemm`` (qtts/quant/kernels.py:89-177);
* ``"library"`` -- ``qtts_b200.quant.kernels.w8_gemm``, the one-file swap of
  qtts/quant/kernels.py described in INTEGRATION.md (``int8.py`` binds
  ``w8_gemm`` and ``kernel_available`` at import, int8.py:37, so the in-process
  form of the swap rebinds those two names);
* ``"eager"`` -- the reference's dequantize-then-matmul expression
  ``F.linear(x, q.to(dtype) * scale[:, None])`` (examples/kernels/tune_w8_gemm.py:73-79).

Weights are random (no checkpoint exists here): linear weights and embeddings
~N(0, 0.02), norm weights 1, biases 0, from a seeded CUDA generator; the slot KV
cache holds 512 earlier positions ~N(0, 1). Attention uses the reference's
``torch_sdpa`` backend in every arm.
"""

from __future__ import annotations

import sys

import torch
import torch.nn.functional as F

from .install import TARGET, installed

BATCH = 8
PRIOR_TOKENS = 512
CODEC_VOCAB = 3072
CODE_VOCAB = 2048
CODEC_EOS = 2150
TTS_PAD = 1000  # text id of the pad embedding (any id inside the small text vocabulary below)


class ReferenceUnavailable(RuntimeError):
    """The reference package is not installed under ``baseline/_ref``."""


def qtts():
    """Import the reference package from ``baseline/_ref``."""
    if not installed():
        raise ReferenceUnavailable(f"reference qtts not installed at {TARGET} (python -m baseline.install)")
    path = str(TARGET)
    if path not in sys.path:
        sys.path.insert(0, path)
    import qtts as ref  # noqa: PLC0415
    import qtts.compilation  # noqa: F401
    import qtts.quant.calibrate  # noqa: F401
    import qtts.quant.int8  # noqa: F401
    import qtts.quant.kernels  # noqa: F401

    if not str(getattr(ref, "__file__", "")).startswith(path):
        raise ReferenceUnavailable(f"a different qtts is already imported ({ref.__file__})")
    return ref


def eager_w8_gemm(x: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor, bias=None) -> torch.Tensor:
    """The reference's naive weight-only expression (examples/kernels/tune_w8_gemm.py:73-79)."""
    return F.linear(x, weight.to(x.dtype) * scale[:, None].to(x.dtype), bias)


def set_kernels(kind: str) -> None:
    """Point the reference's ``Int8WeightOnlyMethod`` at one int8 GEMM (module docstring)."""
    ref = qtts()
    int8 = ref.quant.int8
    if kind == "triton":
        fn, avail = ref.quant.kernels.w8_gemm, ref.quant.kernels.kernel_available
    elif kind == "library":
        from qtts_b200.quant import kernels as lib  # noqa: PLC0415

        fn, avail = lib.w8_gemm, lib.kernel_available
    elif kind == "eager":
        fn, avail = eager_w8_gemm, (lambda: (True, ""))
    else:
        raise ValueError(f"unknown kernel arm {kind!r}")
    int8.w8_gemm = fn
    int8.kernel_available = avail
    # The calibration verdicts are cached by shape only; a new kernel needs new verdicts.
    ref.quant.calibrate.clear_cache()


def hf_config(talker_layers: int = 28, predictor_layers: int = 5):
    """The config-4 model: talker 28 x 2048 (16 q / 8 kv heads of 128, SwiGLU 6144, codec
    vocabulary 3072), code predictor 5 x 1024 (SwiGLU 3072, 16 codebooks of 2048)."""
    qtts()
    from qtts.models.hf_config import CodePredictorHFConfig, Qwen3TTSHFConfig, TalkerHFConfig  # noqa: PLC0415

    cp = CodePredictorHFConfig(
        vocab_size=CODE_VOCAB, hidden_size=1024, intermediate_size=3072, num_hidden_layers=predictor_layers,
        num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
        max_position_embeddings=65536, num_code_groups=16,
    )
    tc = TalkerHFConfig(
        vocab_size=CODEC_VOCAB, hidden_size=2048, intermediate_size=6144, num_hidden_layers=talker_layers,
        num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
        max_position_embeddings=32768, num_code_groups=16, text_hidden_size=2048, text_vocab_size=1024,
        codec_eos_token_id=CODEC_EOS, codec_pad_id=2148, codec_bos_id=2149, codec_think_id=2154,
        codec_nothink_id=2155, codec_think_bos_id=2156, codec_think_eos_id=2157, spk_id={}, spk_is_dialect={},
        codec_language_id={}, code_predictor=cp,
    )
    return Qwen3TTSHFConfig(
        talker=tc, code2wav=None, model_type="qwen3_tts", tts_model_type="custom_voice", tts_model_size="1.7b",
        im_start_token_id=1001, im_end_token_id=1002, tts_pad_token_id=TTS_PAD, tts_bos_token_id=1003,
        tts_eos_token_id=1004,
    )


def runtime_config(batch: int = BATCH):
    qtts()
    from qtts.config import TalkerConfig  # noqa: PLC0415

    return TalkerConfig(
        attention_backend="torch_sdpa", rmsnorm_backend="fused", cuda_graph=True,
        cuda_graph_batch_sizes=(batch,), cuda_graph_key_len_bucket=256, fuse_qkv=True, fuse_gate_up=True,
    )


@torch.no_grad()
def _random_init_(module: torch.nn.Module, gen: torch.Generator) -> None:
    for name, p in module.named_parameters():
        if name.endswith("norm.weight"):
            p.fill_(1.0)
        elif name.endswith(".bias"):
            p.zero_()
        else:
            p.copy_((torch.randn(p.shape, generator=gen, device=p.device) * 0.02).to(p.dtype))


def build_models(*, batch: int = BATCH, quant: str | None = "int8_weight_only", calibrate: bool = False,
                 kernels: str = "library", seed: int = 0, device="cuda", talker_layers: int = 28,
                 predictor_layers: int = 5):
    """(talker, code_predictor, quantization report) built as the reference's engine builds
    them (qtts/engine/engine.py:63-115): modules on the device, weights, the pad embedding,
    then ``apply_quantization`` with ``calibration_batch`` = the batch (max_num_seqs)."""
    ref = qtts()
    from qtts.config import QuantConfig  # noqa: PLC0415
    from qtts.models.code_predictor import CodePredictor  # noqa: PLC0415
    from qtts.models.talker import Qwen3TTSTalker  # noqa: PLC0415

    set_kernels(kernels)
    device = torch.device(device)
    cfg = hf_config(talker_layers, predictor_layers)
    rt = runtime_config(batch)
    talker = Qwen3TTSTalker(cfg, runtime=rt, dtype=torch.bfloat16, device=device, max_num_seqs=batch,
                            max_model_len=768).to(device).eval()
    predictor = CodePredictor(cfg.talker.code_predictor, cfg.talker.hidden_size, runtime=rt,
                              dtype=torch.bfloat16, device=device).to(device).eval()
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    _random_init_(talker, gen)
    _random_init_(predictor, gen)
    talker.init_runtime_buffers()
    report = {}
    if quant is not None:
        report = ref.quant.apply_quantization(
            QuantConfig(method=quant, targets=("talker",), exclude_substrings=(), calibrate=calibrate),
            talker=talker, code_predictor=predictor, calibration_batch=batch,
        )
    cache_gen = torch.Generator(device=device)
    cache_gen.manual_seed(seed + 1)
    with torch.no_grad():
        for t in (talker.cache.k, talker.cache.v):
            prior = torch.randn(t[:, :batch, :PRIOR_TOKENS].shape, generator=cache_gen, device=device)
            t[:, :batch, :PRIOR_TOKENS].copy_(prior.to(t.dtype))
    return talker, predictor, report


def initial_state(batch: int = BATCH, seed: int = 0, device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """(talker hidden state [B, 2048], next-step input embedding [B, 2048]) drawn ~N(0, 1)."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 2)
    hidden = torch.randn((batch, 2048), generator=gen, device=device).to(torch.bfloat16)
    embeds = torch.randn((batch, 2048), generator=gen, device=device).to(torch.bfloat16)
    return hidden, embeds


@torch.inference_mode()
def talker_step_logits(talker, embeds: torch.Tensor) -> torch.Tensor:
    """One eager talker decode step at position 512 for every row, then the masked codec-head
    logits (fp32): ``Qwen3TTSTalker.decode`` + ``logits`` (qtts/models/talker.py:302-356)."""
    rows = embeds.shape[0]
    seq_lens = torch.full((rows,), PRIOR_TOKENS, dtype=torch.long, device=embeds.device)
    hidden = talker.decode(embeds, seq_lens, PRIOR_TOKENS + 1)
    return talker.logits(hidden)


class RefFrame:
    """The reference engine's greedy frame over one batch, replayed from its own CUDA graphs."""

    def __init__(self, talker, predictor, batch: int = BATCH, seed: int = 0) -> None:
        ref = qtts()
        self.talker, self.predictor, self.batch = talker, predictor, batch
        self.graphs = ref.compilation.TalkerDecodeGraphs(talker, (batch,), key_len_bucket=256)
        self.pgraphs = ref.compilation.CodePredictorGraphs(predictor, (batch,), batch)
        self.hidden, self.embeds = initial_state(batch, seed, talker.device)
        self.seq_lens = [PRIOR_TOKENS] * batch
        self.active = [True] * batch
        stacked = predictor.stacked_embedding_weight()
        self.residual = stacked
        self.row_index = torch.arange(stacked.shape[0], device=talker.device).unsqueeze(0).expand(batch, -1)

    @torch.inference_mode()
    def step(self) -> torch.Tensor:
        """One frame; returns the graph's ``[B, 16]`` codes (valid until the next frame)."""
        talker = self.talker
        logits = talker.logits(self.hidden)
        layer0 = logits.argmax(dim=-1)
        layer0_embed = talker.embed_codec(layer0.reshape(-1, 1)).squeeze(1)
        codes = self.pgraphs.run(layer0, layer0_embed, self.hidden, do_sample=False, temperature=0.9, top_k=50)
        gathered = self.residual[self.row_index, codes[:, 1:]]
        next_embeds = layer0_embed + gathered.sum(dim=1) + talker.tts_pad_embed.to(talker.dtype)
        self.hidden = self.graphs.run(next_embeds, self.seq_lens, self.active, PRIOR_TOKENS + 1)
        return codes

    def frames_per_s(self, reps: int = 20, windows: int = 5) -> tuple[float, float]:
        """(frames/s, ms per frame): median of ``windows`` CUDA-event windows of ``reps`` frames
        each, after the graphs are captured; frames/s = batch / frame time."""
        for _ in range(3):
            self.step()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        times = []
        for _ in range(windows):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                self.step()
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / reps)
        ms = sorted(times)[len(times) // 2]
        return self.batch / (ms * 1e-3), ms
