"""Random-init talker decode step + code predictor: the frames/s workload of the benchmark.

This is the end-to-end setting the quantized linears serve (the decode loop of
qtts/models/talker.py and qtts/models/code_predictor.py), reduced to what
drives its cost: every projection is a :class:`LinearBase`, so the library's
quant methods attach to it exactly as they attach to the reference's layers.
Weights are random (no checkpoint is available): ~N(0, 0.02), norms = 1.

One frame, for a batch of B streams:

* talker decode step (28 layers, hidden 2048, 16 query / 8 key-value heads of
  128, per-head RMSNorm on q and k, rotary positions, SwiGLU 6144) over a slot
  KV cache holding 512 earlier tokens; final norm and the codec head
  2048 -> 3072 with the logits masked to [1, 2048) and {2150}; greedy code 0;
* code predictor (5 layers, hidden 1024, the same head layout, SwiGLU 3072):
  the talker's hidden state through small_to_mtp (2048 -> 1024) and the
  embedding of code 0 start a prefix; each of the 15 codebook steps runs the
  5 layers over the whole prefix (2..16 tokens, so its linears see M = B * 2
  .. B * 16 rows), applies that step's head (1024 -> 2048), takes the greedy
  code and appends its embedding.

All shapes are static, so a whole frame is captured in one CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from .layers.linear import LinearBase


@dataclass(frozen=True)
class Dims:
    layers: int
    hidden: int
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 6144


TALKER = Dims(layers=28, hidden=2048, inter=6144)
PREDICTOR = Dims(layers=5, hidden=1024, inter=3072)
CODEC_VOCAB = 3072
CODE_VOCAB = 2048
CODEBOOKS = 16  # code 0 from the talker + 15 from the code predictor
PRIOR_TOKENS = 512


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return F.rms_norm(x, (x.shape[-1],), weight, eps)


def rope_tables(positions: torch.Tensor, dim: int, theta: float = 1.0e6) -> tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / theta ** (torch.arange(0, dim, 2, device=positions.device, dtype=torch.float32) / dim)
    ang = positions.float()[:, None] * inv[None, :]
    return torch.cos(ang), torch.sin(ang)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    # x [B, heads, T, D]; cos/sin [T, D/2]; rotate the two halves.
    x1, x2 = x.float().chunk(2, dim=-1)
    c, s = cos[None, None], sin[None, None]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1).to(x.dtype)


class Block(nn.Module):
    #: Run the input / post-attention norms and SiLU·up inside the quantized
    #: linears that consume them (LinearBase.forward_rmsnorm / forward_silu_mul;
    #: a no-op for unquantized layers). False keeps them as separate torch ops.
    fuse_prologues = True

    def __init__(self, d: Dims, dtype: torch.dtype, device) -> None:
        super().__init__()
        self.d = d
        q, kv = d.heads * d.head_dim, d.kv_heads * d.head_dim
        self.input_norm = nn.Parameter(torch.ones(d.hidden, dtype=dtype, device=device), requires_grad=False)
        self.qkv_proj = LinearBase(d.hidden, q + 2 * kv, dtype=dtype, device=device)
        self.q_norm = nn.Parameter(torch.ones(d.head_dim, dtype=dtype, device=device), requires_grad=False)
        self.k_norm = nn.Parameter(torch.ones(d.head_dim, dtype=dtype, device=device), requires_grad=False)
        self.o_proj = LinearBase(q, d.hidden, dtype=dtype, device=device)
        self.post_norm = nn.Parameter(torch.ones(d.hidden, dtype=dtype, device=device), requires_grad=False)
        self.gate_up_proj = LinearBase(d.hidden, 2 * d.inter, dtype=dtype, device=device)
        self.down_proj = LinearBase(d.inter, d.hidden, dtype=dtype, device=device)

    def _qkv(self, x: torch.Tensor, cos, sin):
        b, t, _ = x.shape
        d = self.d
        if self.fuse_prologues:
            qkv = self.qkv_proj.forward_rmsnorm(x, self.input_norm)
        else:
            qkv = self.qkv_proj(rms_norm(x, self.input_norm))
        q, k, v = qkv.split([d.heads * d.head_dim, d.kv_heads * d.head_dim, d.kv_heads * d.head_dim], dim=-1)
        q = rms_norm(q.view(b, t, d.heads, d.head_dim), self.q_norm).transpose(1, 2)
        k = rms_norm(k.view(b, t, d.kv_heads, d.head_dim), self.k_norm).transpose(1, 2)
        v = v.view(b, t, d.kv_heads, d.head_dim).transpose(1, 2)
        return apply_rope(q, cos, sin), apply_rope(k, cos, sin), v

    def _mlp(self, h: torch.Tensor) -> torch.Tensor:
        if self.fuse_prologues:
            gate_up = self.gate_up_proj.forward_rmsnorm(h, self.post_norm)
            return h + self.down_proj.forward_silu_mul(gate_up)
        gate, up = self.gate_up_proj(rms_norm(h, self.post_norm)).chunk(2, dim=-1)
        return h + self.down_proj(F.silu(gate) * up)

    def decode(self, x: torch.Tensor, cache_k: torch.Tensor, cache_v: torch.Tensor, pos: int, cos, sin):
        """One token per stream at position ``pos`` over the slot cache [B, kv_heads, slots, D]."""
        b = x.shape[0]
        q, k, v = self._qkv(x, cos, sin)
        cache_k[:, :, pos : pos + 1] = k
        cache_v[:, :, pos : pos + 1] = v
        att = F.scaled_dot_product_attention(q, cache_k[:, :, : pos + 1], cache_v[:, :, : pos + 1], enable_gqa=True)
        h = x + self.o_proj(att.transpose(1, 2).reshape(b, 1, -1))
        return self._mlp(h)

    def prefix(self, x: torch.Tensor, cos, sin) -> torch.Tensor:
        """Causal attention over the whole (short) sequence, no cache."""
        b, t, _ = x.shape
        q, k, v = self._qkv(x, cos, sin)
        att = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        h = x + self.o_proj(att.transpose(1, 2).reshape(b, t, -1))
        return self._mlp(h)


class Talker(nn.Module):
    def __init__(self, batch: int, dtype=torch.bfloat16, device="cuda", layers: int = TALKER.layers,
                 seed: int = 0) -> None:
        super().__init__()
        d = Dims(layers=layers, hidden=TALKER.hidden, inter=TALKER.inter)
        self.d = d
        self.layers = nn.ModuleList([Block(d, dtype, device) for _ in range(layers)])
        self.norm = nn.Parameter(torch.ones(d.hidden, dtype=dtype, device=device), requires_grad=False)
        self.codec_head = LinearBase(d.hidden, CODEC_VOCAB, dtype=dtype, device=device)
        slots = 768  # key length 513 bucketed, as the reference's graphs do
        shape = (layers, batch, d.kv_heads, slots, d.head_dim)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.cache_k = torch.randn(shape, generator=gen, device=device).to(dtype)
        self.cache_v = torch.randn(shape, generator=gen, device=device).to(dtype)
        mask = torch.full((CODEC_VOCAB,), float("-inf"), device=device)
        mask[1:2048] = 0.0
        mask[2150] = 0.0
        self.logit_mask = mask
        self.pos = PRIOR_TOKENS
        self.cos, self.sin = rope_tables(torch.tensor([self.pos], device=device), d.head_dim)

    def step(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """x [B, hidden] -> (last hidden [B, hidden], greedy code 0 [B])."""
        h = x[:, None, :]
        for i, layer in enumerate(self.layers):
            h = layer.decode(h, self.cache_k[i], self.cache_v[i], self.pos, self.cos, self.sin)
        h = rms_norm(h[:, 0], self.norm)
        logits = self.codec_head(h).float() + self.logit_mask
        return h, logits.argmax(dim=-1)


def _fused_head_ok(head: LinearBase, k: int) -> bool:
    """Whether a codebook head runs as the library's fused head (norm, int8 head, argmax and
    the next step's embedding in one launch): an int8 weight-only head of a width it takes."""
    from .quant.int8 import Int8WeightOnlyMethod

    return isinstance(head.quant_method, Int8WeightOnlyMethod) and k % 128 == 0 and k <= 2048


class CodePredictor(nn.Module):
    #: End each codebook step with the library's fused head (qtts_w8a16_head_argmax: the
    #: final norm, the int8 head, the greedy argmax and the next step's embedding row in one
    #: launch) when the head is int8; False keeps head, argmax and lookup as separate ops.
    fuse_heads = True

    def __init__(self, dtype=torch.bfloat16, device="cuda", layers: int = PREDICTOR.layers,
                 codebooks: int = CODEBOOKS - 1, seed: int = 0) -> None:
        super().__init__()
        d = Dims(layers=layers, hidden=PREDICTOR.hidden, inter=PREDICTOR.inter)
        self.d = d
        self.codebooks = codebooks
        self.small_to_mtp_projection = LinearBase(TALKER.hidden, d.hidden, dtype=dtype, device=device)
        self.layers = nn.ModuleList([Block(d, dtype, device) for _ in range(layers)])
        self.norm = nn.Parameter(torch.ones(d.hidden, dtype=dtype, device=device), requires_grad=False)
        self.lm_head = nn.ModuleList([LinearBase(d.hidden, CODE_VOCAB, dtype=dtype, device=device)
                                      for _ in range(codebooks)])
        # Embeddings of code 0 (from the talker's codec vocabulary) and of codes 1..15.
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        self.embed = nn.ParameterList(
            [nn.Parameter((torch.randn(CODEC_VOCAB if i == 0 else CODE_VOCAB, d.hidden, generator=gen,
                                       device=device) * 0.02).to(dtype), requires_grad=False)
             for i in range(codebooks)])
        self.cos, self.sin = rope_tables(torch.arange(codebooks + 1, device=device), d.head_dim)

    def run(self, talker_hidden: torch.Tensor, code0: torch.Tensor) -> torch.Tensor:
        """Greedy codes 1..codebooks [B, codebooks] for each stream."""
        seq = [self.small_to_mtp_projection(talker_hidden), self.embed[0][code0]]
        codes = []
        for s in range(self.codebooks):
            x = torch.stack(seq, dim=1)  # [B, s + 2, hidden]
            t = x.shape[1]
            for layer in self.layers:
                x = layer.prefix(x, self.cos[:t], self.sin[:t])
            head = self.lm_head[s]
            if self.fuse_heads and _fused_head_ok(head, x.shape[-1]):
                from .quant import kernels as qk

                nxt = self.embed[s + 1] if s + 1 < self.codebooks else None
                code, emb = qk.w8_head_argmax(x[:, -1], head.int8_weight, head.int8_scale, norm_weight=self.norm,
                                              embed=nxt)
                codes.append(code)
                if emb is not None:
                    seq.append(emb)
                continue
            if Block.fuse_prologues:
                code = self.lm_head[s].forward_rmsnorm(x[:, -1], self.norm).float().argmax(dim=-1)
            else:
                code = self.lm_head[s](rms_norm(x[:, -1], self.norm)).float().argmax(dim=-1)
            codes.append(code)
            if s + 1 < self.codebooks:
                seq.append(self.embed[s + 1][code])
        return torch.stack(codes, dim=1)


def random_init_(module: nn.Module, seed: int) -> None:
    """Every linear weight ~N(0, 0.02), drawn on the device from a seeded generator."""
    gen = None
    for m in module.modules():
        if isinstance(m, LinearBase):
            if gen is None:
                gen = torch.Generator(device=m.weight.device)
                gen.manual_seed(seed)
            w = torch.randn(m.weight.shape, generator=gen, device=m.weight.device) * 0.02
            m.weight.data.copy_(w.to(m.weight.dtype))


class Frame:
    """Talker step + code predictor for a batch of streams, capturable as one CUDA graph."""

    def __init__(self, batch: int = 8, *, device="cuda", talker_layers: int = TALKER.layers,
                 predictor_layers: int = PREDICTOR.layers, codebooks: int = CODEBOOKS - 1, seed: int = 0) -> None:
        self.batch = batch
        self.talker = Talker(batch, device=device, layers=talker_layers, seed=seed + 3)
        self.predictor = CodePredictor(device=device, layers=predictor_layers, codebooks=codebooks, seed=seed + 4)
        random_init_(self.talker, seed)
        random_init_(self.predictor, seed + 1)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + 2)
        self.x = torch.randn((batch, TALKER.hidden), generator=gen, device=device).to(torch.bfloat16)
        self.codes = torch.zeros((batch, codebooks + 1), dtype=torch.int64, device=device)
        self.graph: torch.cuda.CUDAGraph | None = None

    @torch.no_grad()
    def run(self) -> torch.Tensor:
        h, code0 = self.talker.step(self.x)
        rest = self.predictor.run(h, code0)
        self.codes[:, 0] = code0
        self.codes[:, 1:] = rest
        return self.codes

    @torch.no_grad()
    def capture(self) -> None:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.run()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.run()
        torch.cuda.synchronize()

    def frame_weight_bytes(self) -> int:
        """Linear-weight bytes one frame reads: the talker once, the predictor once per codebook
        step (its 15 heads once in total)."""
        def nbytes(mod: nn.Module) -> int:
            total = 0
            for m in mod.modules():
                if isinstance(m, LinearBase):
                    total += sum(t.numel() * t.element_size() for t in (
                        getattr(m, "int8_weight", None), m.weight) if t is not None)
            return total
        pred_layers = sum(nbytes(layer) for layer in self.predictor.layers)
        heads = sum(nbytes(h) for h in self.predictor.lm_head)
        return nbytes(self.talker) + self.predictor.codebooks * pred_layers + heads + nbytes(
            self.predictor.small_to_mtp_projection)


def timed_frames_per_s(frame: Frame, reps: int = 20, windows: int = 5) -> tuple[float, float]:
    """(frames/s, ms per frame step): the median over ``windows`` timing windows of ``reps``
    graph replays each (one window alone has read 10-15 % fast or slow on a shared box);
    frames/s = batch / step time."""
    if frame.graph is None:
        frame.capture()
    stream = torch.cuda.current_stream()
    frame.graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(windows):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            frame.graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / reps)
    ms = sorted(times)[len(times) // 2]
    return frame.batch / (ms * 1e-3), ms
