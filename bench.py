#!/usr/bin/env python
"""Benchmark of the int8 weight-only (W8A16) hot path on B200.

Workload (the configuration the headline metric is
quoted on): the talker's four linear shapes -- fused qkv 4096x2048, o_proj
2048x2048, gate_up 12288x2048, down 2048x6144 -- at M in {1,2,4,8,16,32,64},
weights fp32 ~N(0, 0.02) quantized per output row to int8 (bf16 scales, as
Int8WeightOnlyMethod stores them), activations bf16 ~N(0, 1), seed 0.

One step = the sweep at the reference benchmark's own call count: every
(shape, M) point runs 2016 calls (the reference times 10 calls x 200 replays
per point, examples/kernels/tune_w8_gemm.py:48-70), as 9 replays of a CUDA
graph of 224 calls through ``qtts_b200.quant.kernels.w8_gemm``. Each call
reads a different copy of the weight: per shape a pool of at least 256 MB
(> 2x the 126 MB L2), reused only after a full pool, so every call streams its
weights from HBM.

``value`` = algorithmic bytes of all calls (int8 W + bf16 scale + bf16 x +
bf16 out) / device time, aggregated over ranks; ``e2e`` is the same sweep with
every call copying its x in from pinned host memory and its output back out. ``--impl reference`` times the reference's eager CPU path
(``F.linear(x, q.to(bf16) * scale)``, restated in ``oracle/``) on the host
cores instead.

Multi-GPU: one process per GPU under torchrun; each rank runs the full sweep
on its own GPU (independent replicas, weak scaling), timing is the max over
ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "tts-inference_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

SHAPES = [("qkv", 4096, 2048), ("o_proj", 2048, 2048), ("gate_up", 12288, 2048), ("down_proj", 2048, 6144)]
ROWS = (1, 2, 4, 8, 16, 32, 64)
CALLS_PER_GRAPH = 224  # multiple of every pool size below
REPLAYS_PER_POINT = 9  # 9 x 224 = 2016 calls per point (--replays)
POOL_MIN_BYTES = 256 << 20
METRIC = "int8 W8A16 GEMM HBM GB/s (talker linear sweep, M=1..64)"
# DRAM bytes per launch of the dominant kernel (skinny_w8a16_kernel, down_proj
# M=1) from one `ncu --set full` capture of that launch:
# dram__bytes_read.sum + dram__bytes_write.sum, against its algorithmic bytes.
NCU_TRAFFIC = {"case": "down_proj 2048x6144, M=1", "bytes_per_launch": 12666624, "algorithmic_bytes": 12603392}


def algo_bytes(n: int, k: int, m: int) -> int:
    """Algorithmic bytes of one call: int8 weight, bf16 scale, bf16 x, bf16 out."""
    return n * k + 2 * n + 2 * m * k + 2 * m * n


def pool_size(n: int, k: int) -> int:
    """Smallest divisor of CALLS_PER_GRAPH whose copies hold >= POOL_MIN_BYTES."""
    need = -(-POOL_MIN_BYTES // (n * k))
    for d in range(1, CALLS_PER_GRAPH + 1):
        if CALLS_PER_GRAPH % d == 0 and d >= need:
            return d
    return CALLS_PER_GRAPH


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
        "clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, device_index: int, log_path: Path | None = None):
        self.device_index = device_index
        self.lines: list[str] = []
        self.proc = None
        self.log_path = log_path
        self._thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.device_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            self.proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()

    def _read(self):
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=2)
        sm, sm_max, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if self.log_path is not None:
            self.log_path.write_text("\n".join(self.lines) + "\n")
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(sm_max) if sm_max else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ----------------------------------------------------------------------------- distributed


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(world, value: float) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU reference arm


def cpu_port_sample(budget_s: float, rows=ROWS) -> dict:
    """The reference's eager dequant-then-matmul on host cores (oracle port)."""
    import oracle.cpu_baseline as cb

    return cb.time_sweep(SHAPES, rows, budget_s=budget_s)


def run_reference_arm(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle.cpu_baseline as cb

    threads = cb.use_all_threads()
    work = cb.SweepWork(SHAPES, ROWS, seed=0)
    for _ in range(args.warmup):
        work.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        work.step()
    elapsed = time.perf_counter() - t0
    bytes_per_step = work.bytes_per_step
    value = bytes_per_step * args.steps / elapsed / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {
            "workload": "config-2 talker linear sweep on the host CPU: 4 shapes x M in {1,2,4,8,16,32,64}, "
            "one call per point per step (a bounded sample of the GPU step's 2016 calls per point)",
        },
        "cpu_baseline": {
            "value": value,
            "unit": "GB/s",
            "cores": threads,
            "kind": "port",
            "sample": "one eager F.linear(x, q.to(bf16) * scale[:, None]) per (shape, M) point per step",
        },
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm


class Point:
    def __init__(self, label, n, k, m):
        self.label, self.n, self.k, self.m = label, n, k, m
        self.bytes = algo_bytes(n, k, m)
        self.graph = None
        self.e2e_graph = None
        self.bf16_graph = None


def build_pools(device, seed: int):
    from qtts_b200.quant import kernels as qk

    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    pools = {}
    for label, n, k in SHAPES:
        p = pool_size(n, k)
        qs = torch.empty((p, n, k), dtype=torch.int8, device=device)
        ss = torch.empty((p, n), dtype=torch.bfloat16, device=device)
        for i in range(p):
            w = torch.randn((n, k), generator=gen, device=device) * 0.02
            q, s = qk.quantize_int8_rows(w)
            qs[i].copy_(q)
            ss[i].copy_(s.to(torch.bfloat16))
            del w, q, s
        pools[label] = (qs, ss)
    torch.cuda.synchronize()
    return pools


def capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


FP8_ROWS = (16, 32, 64, 128)


def graph_us_per_call(fn, reps=3) -> float:
    """Capture ``fn`` (CALLS_PER_GRAPH calls) in a CUDA graph, replay it once
    untimed and ``reps`` times between CUDA events; microseconds per call."""
    stream = torch.cuda.current_stream()
    g = capture(fn)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g.replay()
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * CALLS_PER_GRAPH)


def fp8_algo_bytes(n: int, k: int, m: int) -> int:
    """Config-3 bytes of one fp8 linear: e4m3 W + fp32 scale, bf16 x in, e4m3 x + fp32 scale
    out and back in (the separate quantization step), bf16 out."""
    return n * k + 4 * n + 2 * m * k + 2 * (m * k + 4 * m) + 2 * m * n


def fp8_sweep(device, seed: int) -> dict:
    """Config 3: the fp8 W8A8 path (per-token activation quantization + tcgen05 scaled GEMM,
    as Fp8Method.apply runs it) on the four talker shapes at M in {16, 32, 64, 128}, beside
    the reference's own op sequence on the same GPU (torch amax/clamp/div/cast +
    torch._scaled_mm). Weight copies rotate through >= 256 MB per shape, as in config 2."""
    from qtts_b200.quant import kernels as qk

    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 7)
    out: dict = {}
    timed = graph_us_per_call

    tot_bytes = tot_us = tot_ref_us = 0.0
    for label, n, k in SHAPES:
        p = pool_size(n, k)
        wq = torch.empty((p, n, k), dtype=torch.float8_e4m3fn, device=device)
        ws = torch.empty((p, n), dtype=torch.float32, device=device)
        for i in range(p):
            w = torch.randn((n, k), generator=gen, device=device) * 0.02
            q, s = qk.quantize_fp8_rows(w)
            wq[i].copy_(q)
            ws[i].copy_(s)
            del w, q, s
        wt = [wq[i].t() for i in range(p)]  # the reference's column-major fp8_weight views
        for m in FP8_ROWS:
            x = torch.randn((m, k), generator=gen, device=device).to(torch.bfloat16)

            def ours(x=x):
                for c in range(CALLS_PER_GRAPH):
                    xq, sx = qk.fp8_quant_rows(x)
                    qk.fp8_scaled_mm(xq, sx, wq[c % p], ws[c % p], None, torch.bfloat16)

            def reference(x=x):
                for c in range(CALLS_PER_GRAPH):
                    sx = x.abs().amax(dim=1, keepdim=True).clamp_min(1e-6).float() / 448.0
                    xq = (x.float() / sx).to(torch.float8_e4m3fn)
                    torch._scaled_mm(xq, wt[c % p], scale_a=sx, scale_b=ws[c % p].reshape(1, -1),
                                     bias=None, out_dtype=torch.bfloat16)

            # The GEMM alone on the same quantized activations: the library's scaled GEMM
            # against torch._scaled_mm (cuBLASLt), the call Fp8Method.apply makes.
            xq0, sx0 = qk.fp8_quant_rows(x)

            def ours_gemm(xq0=xq0, sx0=sx0):
                for c in range(CALLS_PER_GRAPH):
                    qk.fp8_scaled_mm(xq0, sx0, wq[c % p], ws[c % p], None, torch.bfloat16)

            def scaled_mm_gemm(xq0=xq0, sx0=sx0):
                for c in range(CALLS_PER_GRAPH):
                    torch._scaled_mm(xq0, wt[c % p], scale_a=sx0.reshape(-1, 1), scale_b=ws[c % p].reshape(1, -1),
                                     bias=None, out_dtype=torch.bfloat16)

            us = timed(ours)
            gemm_us = timed(ours_gemm)
            try:
                ref_us = timed(reference)
                smm_us = timed(scaled_mm_gemm)
            except Exception as exc:  # _scaled_mm unavailable for this layout/build
                ref_us = smm_us = None
                print(f"torch._scaled_mm reference failed: {exc}", file=sys.stderr)
            b = fp8_algo_bytes(n, k, m)
            out.setdefault(label, {})[str(m)] = {
                "us": round(us, 3),
                "gbs": round(b / (us * 1e-6) / 1e9, 1),
                "tflops": round(2 * m * n * k / (us * 1e-6) / 1e12, 1),
                "torch_us": round(ref_us, 3) if ref_us else None,
                "speedup_vs_torch": round(ref_us / us, 3) if ref_us else None,
                "gemm_us": round(gemm_us, 3),
                "scaled_mm_us": round(smm_us, 3) if smm_us else None,
                "speedup_vs_scaled_mm": round(smm_us / gemm_us, 3) if smm_us else None,
            }
            tot_bytes += b
            tot_us += us
            tot_ref_us += ref_us or 0.0
        del wq, ws, wt
        torch.cuda.empty_cache()
    return {
        "workload": "config 3: fp8 e4m3 W8A8 (act quant + tcgen05 scaled GEMM, 2 launches per linear) on the "
        "4 talker shapes at M in {16,32,64,128}; weights rotate through >= 256 MB per shape",
        "gbs": round(tot_bytes / (tot_us * 1e-6) / 1e9, 1),
        "torch_gbs": round(tot_bytes / (tot_ref_us * 1e-6) / 1e9, 1) if tot_ref_us else None,
        "per_point": out,
    }


def w8a8_sweep(device, seed: int) -> dict:
    """int8 W8A8 (Int8Method.apply: per-token int8 activation quantization + tcgen05
    kind::i8 GEMM) on the four talker shapes at M in {16, 32, 64, 128}, beside the
    reference's op sequence on the same GPU (torch amax/clamp/div/round/clamp/cast,
    torch._int_mm with its 17-row padding, the fp32 scaling). Same bytes as config 3.
    Weights rotate through >= 256 MB per shape."""
    from qtts_b200.quant import kernels as qk

    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 13)
    out: dict = {}
    tot_bytes = tot_us = tot_ref_us = 0.0
    for label, n, k in SHAPES:
        p = pool_size(n, k)
        wq = torch.empty((p, n, k), dtype=torch.int8, device=device)
        ws = torch.empty((p, n), dtype=torch.float32, device=device)
        for i in range(p):
            q, s = qk.quantize_int8_rows(torch.randn((n, k), generator=gen, device=device) * 0.02)
            wq[i].copy_(q)
            ws[i].copy_(s)
            del q, s
        wkn = torch.empty((p, k, n), dtype=torch.int8, device=device)
        for i in range(p):
            wkn[i].copy_(wq[i].t())  # the reference's [K, N] int8_weight (int8.py:126-128)
        for m in FP8_ROWS:
            x = torch.randn((m, k), generator=gen, device=device).to(torch.bfloat16)

            def ours(x=x):
                for c in range(CALLS_PER_GRAPH):
                    xq, sx = qk.int8_quant_rows(x)
                    qk.i8_scaled_mm(xq, sx, wq[c % p], ws[c % p], None, torch.bfloat16)

            def reference(x=x, m=m):
                for c in range(CALLS_PER_GRAPH):
                    scale_x = x.abs().amax(dim=1, keepdim=True).clamp_min(1e-6) / 127.0
                    q = (x / scale_x).round().clamp_(-127, 127).to(torch.int8)
                    if m < 17:
                        q = torch.cat([q, q.new_zeros(17 - m, k)], dim=0)
                    acc = torch._int_mm(q, wkn[c % p])[:m]
                    (acc.float() * scale_x.float() * ws[c % p].reshape(1, -1)).to(torch.bfloat16)

            us = graph_us_per_call(ours)
            try:
                ref_us = graph_us_per_call(reference)
            except Exception as exc:  # torch._int_mm unavailable for this shape/build
                ref_us = None
                print(f"torch._int_mm reference failed: {exc}", file=sys.stderr)
            b = fp8_algo_bytes(n, k, m)
            out.setdefault(label, {})[str(m)] = {
                "us": round(us, 3),
                "gbs": round(b / (us * 1e-6) / 1e9, 1),
                "torch_us": round(ref_us, 3) if ref_us else None,
                "speedup_vs_torch": round(ref_us / us, 3) if ref_us else None,
            }
            tot_bytes += b
            tot_us += us
            tot_ref_us += ref_us or 0.0
        del wq, ws, wkn
        torch.cuda.empty_cache()
    return {
        "workload": "int8 W8A8 (act quant + tcgen05 kind::i8 GEMM, 2 launches per linear) on the 4 talker shapes "
        "at M in {16,32,64,128}; weights rotate through >= 256 MB per shape",
        "gbs": round(tot_bytes / (tot_us * 1e-6) / 1e9, 1),
        "torch_gbs": round(tot_bytes / (tot_ref_us * 1e-6) / 1e9, 1) if tot_ref_us else None,
        "per_point": out,
    }


HEADS, HEAD_N, HEAD_K, HEAD_ROWS = 15, 2048, 1024, 8


def grouped_heads(device, seed: int) -> dict:
    """Config 5's second part: the code predictor's 15 codebook heads (lm_head[i] 1024 -> 2048,
    qtts/models/code_predictor.py:159-161, 235) as int8 W8A16 at M = 8 rows per head: one
    grouped launch (qtts_w8a16_grouped_gemm) against 15 separate library calls and against
    cuBLAS bf16 (torch.bmm over the stacked heads, and 15 F.linear calls); plus the engine's
    form, one head per call chosen by a device index (the heads run one per sequential step,
    so a graph of one step serves every step). Stacked weights rotate through >= 256 MB."""
    import torch.nn.functional as F

    from qtts_b200.quant import kernels as qk

    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 19)
    g_, n, k, m = HEADS, HEAD_N, HEAD_K, HEAD_ROWS
    p = pool_size(g_ * n, k)
    wq = torch.empty((p, g_ * n, k), dtype=torch.int8, device=device)
    ws = torch.empty((p, g_ * n), dtype=torch.bfloat16, device=device)
    wb = torch.empty((p, g_, n, k), dtype=torch.bfloat16, device=device)
    for i in range(p):
        w = torch.randn((g_ * n, k), generator=gen, device=device) * 0.02
        q, s_ = qk.quantize_int8_rows(w)
        wq[i].copy_(q)
        ws[i].copy_(s_.to(torch.bfloat16))
        wb[i].copy_(w.view(g_, n, k).to(torch.bfloat16))
        del w, q, s_
    x = torch.randn((g_, m, k), generator=gen, device=device).to(torch.bfloat16)
    index = torch.full((1,), 7, dtype=torch.int64, device=device)

    def grouped():
        for c in range(CALLS_PER_GRAPH):
            qk.w8_grouped_gemm(x, wq[c % p], ws[c % p])

    def separate():
        for c in range(CALLS_PER_GRAPH):
            for h in range(g_):
                qk.w8_gemm(x[h], wq[c % p, h * n:(h + 1) * n], ws[c % p, h * n:(h + 1) * n])

    def indexed():
        for c in range(CALLS_PER_GRAPH):
            qk.w8_indexed_gemm(x[0], wq[c % p], ws[c % p], index, g_)

    def bf16_bmm():
        for c in range(CALLS_PER_GRAPH):
            torch.bmm(x, wb[c % p].transpose(1, 2))

    def bf16_separate():
        for c in range(CALLS_PER_GRAPH):
            for h in range(g_):
                F.linear(x[h], wb[c % p, h])

    us = {name: graph_us_per_call(fn) for name, fn in (("grouped", grouped), ("separate", separate),
                                                       ("indexed", indexed), ("bf16_bmm", bf16_bmm),
                                                       ("bf16_separate", bf16_separate))}
    all_bytes = g_ * n * k + 2 * g_ * n + 2 * g_ * m * k + 2 * g_ * m * n
    one_bytes = n * k + 2 * n + 2 * m * k + 2 * m * n
    del wq, ws, wb
    torch.cuda.empty_cache()
    return {
        "workload": f"{g_} codebook heads {n}x{k} int8 W8A16, M = {m} rows per head; weights rotate through "
        ">= 256 MB",
        "grouped_us": round(us["grouped"], 3),
        "grouped_gbs": round(all_bytes / (us["grouped"] * 1e-6) / 1e9, 1),
        "separate_us": round(us["separate"], 3),
        "bf16_bmm_us": round(us["bf16_bmm"], 3),
        "bf16_separate_us": round(us["bf16_separate"], 3),
        "speedup_vs_separate": round(us["separate"] / us["grouped"], 3),
        "speedup_vs_bf16_bmm": round(us["bf16_bmm"] / us["grouped"], 3),
        "indexed_one_head_us": round(us["indexed"], 3),
        "indexed_one_head_gbs": round(one_bytes / (us["indexed"] * 1e-6) / 1e9, 1),
    }


PROLOGUE_ROWS = (1, 8, 16, 64)


def prologue_sweep(device, seed: int) -> dict:
    """Fused activation prologues: the talker's input / post-attention RMSNorm feeding qkv /
    gate_up, and SiLU·up feeding down_proj (qtts/models/talker.py:249, 271;
    qtts/layers/activation.py:147), as one library call (qtts_w8a16_gemm_prologue) beside
    the same prologue as torch ops ahead of the library's plain GEMM, at M in {1, 8, 16,
    64}. Weights rotate through >= 256 MB per shape."""
    import torch.nn.functional as F

    from qtts_b200.quant import kernels as qk

    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 17)
    cases = [("rmsnorm+qkv", 4096, 2048, "rms"), ("rmsnorm+gate_up", 12288, 2048, "rms"),
             ("silu_mul+down_proj", 2048, 6144, "silu")]
    out: dict = {}
    tot_fused = tot_torch = 0.0
    for label, n, k, kind in cases:
        p = pool_size(n, k)
        qs = torch.empty((p, n, k), dtype=torch.int8, device=device)
        ss = torch.empty((p, n), dtype=torch.bfloat16, device=device)
        for i in range(p):
            q, s_ = qk.quantize_int8_rows(torch.randn((n, k), generator=gen, device=device) * 0.02)
            qs[i].copy_(q)
            ss[i].copy_(s_.to(torch.bfloat16))
            del q, s_
        nw = (1 + 0.1 * torch.randn(k, generator=gen, device=device)).to(torch.bfloat16)
        for m in PROLOGUE_ROWS:
            width = k if kind == "rms" else 2 * k
            x = torch.randn((m, width), generator=gen, device=device).to(torch.bfloat16)
            if kind == "rms":
                def fused(x=x):
                    for c in range(CALLS_PER_GRAPH):
                        qk.w8_gemm_rmsnorm(x, nw, 1e-6, qs[c % p], ss[c % p])

                def torch_prologue(x=x):
                    for c in range(CALLS_PER_GRAPH):
                        qk.w8_gemm(F.rms_norm(x, (k,), nw, 1e-6), qs[c % p], ss[c % p])
            else:
                def fused(x=x):
                    for c in range(CALLS_PER_GRAPH):
                        qk.w8_gemm_silu_mul(x, qs[c % p], ss[c % p])

                def torch_prologue(x=x):
                    for c in range(CALLS_PER_GRAPH):
                        gate, up = x.chunk(2, dim=-1)
                        qk.w8_gemm(F.silu(gate) * up, qs[c % p], ss[c % p])
            xa = x[:, :k].contiguous()

            def gemm_only(xa=xa):
                for c in range(CALLS_PER_GRAPH):
                    qk.w8_gemm(xa, qs[c % p], ss[c % p])

            us, us_t, us_g = graph_us_per_call(fused), graph_us_per_call(torch_prologue), graph_us_per_call(gemm_only)
            out.setdefault(label, {})[str(m)] = {
                "fused_us": round(us, 3),
                "torch_prologue_us": round(us_t, 3),
                "gemm_alone_us": round(us_g, 3),
                "one_launch": qk.prologue_fused(m, n, k, 1 if kind == "rms" else 2),
                "speedup": round(us_t / us, 3),
            }
            tot_fused += us
            tot_torch += us_t
        del qs, ss
        torch.cuda.empty_cache()
    return {
        "workload": "RMSNorm -> qkv / gate_up and SiLU·up -> down_proj (talker shapes) at M in {1,8,16,64}: "
        "one qtts_w8a16_gemm_prologue call vs the torch prologue + the library's GEMM, in CUDA graphs",
        "speedup_overall": round(tot_torch / tot_fused, 3),
        "per_point": out,
    }


def fp8w_sweep(device, seed: int) -> dict:
    """fp8 weight-only (e4m3 weights, bf16 activations, Fp8WeightOnlyMethod.apply) on the
    config-2 grid: the four talker shapes at M in {1..64}, weights rotating through
    >= 256 MB per shape. Beside it, the one route open to the reference, whose
    Fp8WeightOnlyMethod is unimplemented (qtts/quant/fp8.py:92-122): dequantize the
    weight to bf16 in global memory, then F.linear. Bytes per call as config 2 (N*K
    weight bytes, fp32 scale)."""
    from qtts_b200.quant import kernels as qk

    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 11)
    out: dict = {}
    tot_bytes = tot_us = tot_ref_us = 0.0
    for label, n, k in SHAPES:
        p = pool_size(n, k)
        wq = torch.empty((p, n, k), dtype=torch.float8_e4m3fn, device=device)
        ws = torch.empty((p, n), dtype=torch.float32, device=device)
        for i in range(p):
            w = torch.randn((n, k), generator=gen, device=device) * 0.02
            q, s = qk.quantize_fp8_rows(w)
            wq[i].copy_(q)
            ws[i].copy_(s)
            del w, q, s
        for m in ROWS:
            x = torch.randn((m, k), generator=gen, device=device).to(torch.bfloat16)
            y = torch.empty((m, n), dtype=torch.bfloat16, device=device)

            def ours(x=x, y=y):
                for c in range(CALLS_PER_GRAPH):
                    qk.fp8w_gemm(x, wq[c % p], ws[c % p], None, out=y)

            def dequant_linear(x=x):
                for c in range(CALLS_PER_GRAPH):
                    w_bf16 = (wq[c % p].to(torch.float32) * ws[c % p][:, None]).to(torch.bfloat16)
                    torch.nn.functional.linear(x, w_bf16)

            us = graph_us_per_call(ours)
            ref_us = graph_us_per_call(dequant_linear, reps=1)
            b = n * k + 4 * n + 2 * m * k + 2 * m * n
            out.setdefault(label, {})[str(m)] = {
                "us": round(us, 3),
                "gbs": round(b / (us * 1e-6) / 1e9, 1),
                "dequant_linear_us": round(ref_us, 3),
                "speedup": round(ref_us / us, 2),
            }
            tot_bytes += b
            tot_us += us
            tot_ref_us += ref_us
        del wq, ws
        torch.cuda.empty_cache()
    return {
        "workload": "fp8 e4m3 weight-only (one fused launch per linear) on the 4 talker shapes at "
        "M in {1,2,4,8,16,32,64}; weights rotate through >= 256 MB per shape",
        "gbs": round(tot_bytes / (tot_us * 1e-6) / 1e9, 1),
        "dequant_linear_gbs": round(tot_bytes / (tot_ref_us * 1e-6) / 1e9, 1),
        "per_point": out,
    }


SHARD_POINTS = [(k, n, m) for k in (2048, 6144) for n in (12288, 49152) for m in (1, 8, 64)]
SHARD_CALLS = 32
SHARD_PARITY_POINTS = [(2048, 12288, 1), (6144, 12288, 8), (2048, 49152, 64), (6144, 49152, 1)]


def sharded_parity(world: int, rank: int, device, seed: int, k: int, n: int, m: int) -> float:
    """Max relative error (max over ranks, of both the NCCL all-gather form and the fused
    peer-store form) of the gathered [M, N] output against the unsharded library GEMM on the
    same seeded weights; -1.0 when a form failed to run."""
    from qtts_b200.quant import kernels as qk
    from qtts_b200.sharded import FusedAllGatherW8Linear, ShardedW8Linear, shard_rows

    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 101)  # the same full weight on every rank
    w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=device, generator=gen)
    sc = (torch.rand(n, device=device, generator=gen) * 1e-3).to(torch.bfloat16)
    x = torch.randn((m, k), generator=gen, device=device).to(torch.bfloat16)
    full = qk.w8_gemm(x, w, sc).float()
    start, stop = shard_rows(n, world, rank)
    errs = []
    try:
        nccl = ShardedW8Linear(w[start:stop].contiguous(), sc[start:stop].contiguous(), n)(x).float()
        fused = FusedAllGatherW8Linear(w[start:stop].contiguous(), sc[start:stop].contiguous(), n, max_rows=m)
        got = fused(x).float()
        torch.cuda.synchronize()
        scale = full.abs().max().clamp_min(1e-30)
        errs = [((nccl - full).abs().max() / scale).item(), ((got - full).abs().max() / scale).item()]
        del fused
    except Exception:
        errs = [-1.0]
    barrier(world)
    err = max(errs) if errs and min(errs) >= 0 else -1.0
    worst = max_over_ranks(world, err if err >= 0 else 1e9)
    return -1.0 if worst >= 1e9 else worst


def sharded_sweep(world: int, rank: int, device, seed: int) -> dict:
    """Config 5: one int8 weight-only GEMM split along N over the ranks (each rank holds
    ceil(N / world) rows of W and scale), outputs all-gathered over NCCL. The local GEMM and
    the GEMM followed by NCCL's all-gather are each timed in a CUDA graph (and the all-gather
    alone in an eager loop, host launch cost included, for reference), as the max over ranks
    of CUDA-event time; the fused form is one kernel per rank per call. Each point also times
    the unsharded GEMM on one GPU, so ``sharded_efficiency`` = t(1 GPU) / (g x best sharded
    time), and every point's gathered output is checked against the unsharded GEMM."""
    from qtts_b200 import _native as nat
    from qtts_b200.sharded import FusedAllGatherW8Linear, ShardedW8Linear, shard_rows

    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 11)
    stream = torch.cuda.current_stream()
    pk = peaks()
    res: dict = {}

    def time_graph(fn, reps=3):
        g = capture(fn)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g.replay()
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        del g
        return max_over_ranks(world, ms) * 1e3 / SHARD_CALLS

    def time_eager(fn, reps=3):
        fn()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(world, e0.elapsed_time(e1) / reps) * 1e3 / SHARD_CALLS

    fused_ok, fused_error = True, None
    for k, n, m in SHARD_POINTS:
        start, stop = shard_rows(n, world, rank)
        rows = stop - start
        copies = max(1, min(8, -(-POOL_MIN_BYTES // max(1, rows * k))))
        ws = [torch.randint(-127, 128, (rows, k), dtype=torch.int8, device=device, generator=gen)
              for _ in range(copies)]
        ss = [(torch.rand(rows, device=device, generator=gen) * 1e-3).to(torch.bfloat16) for _ in range(copies)]
        lins = [ShardedW8Linear(ws[i], ss[i], n) for i in range(copies)]
        x = torch.randn((m, k), generator=gen, device=device).to(torch.bfloat16)
        block = torch.zeros((m, lins[0].shard), dtype=torch.bfloat16, device=device)
        gathered = torch.empty((world, m, lins[0].shard), dtype=torch.bfloat16, device=device)

        def gemm_only():
            for c in range(SHARD_CALLS):
                lins[c % copies].local(x, block)

        def gather_only():
            for _ in range(SHARD_CALLS):
                lins[0].gather(block, gathered)

        # The fused form: one kernel per rank per call stores its block into every
        # rank's gathered buffer over peer memory (the copies share one buffer set).
        fused = [FusedAllGatherW8Linear(ws[0], ss[0], n, max_rows=m)]
        fused += [FusedAllGatherW8Linear(ws[i], ss[i], n, max_rows=m, share_from=fused[0]) for i in range(1, copies)]

        def fused_calls():
            for c in range(SHARD_CALLS):
                fused[c % copies](x)

        def gemm_gather():
            for c in range(SHARD_CALLS):
                lins[0].gather(lins[c % copies].local(x, block), gathered)

        gemm_us = time_graph(gemm_only)
        gather_us = time_eager(gather_only) if world > 1 else 0.0  # one GPU: the block is the output
        # GEMM + NCCL all-gather captured together (every rank captures the same collectives).
        gemm_gather_graph_us = time_graph(gemm_gather) if world > 1 else gemm_us
        # The unsharded GEMM on this GPU alone: the strong-scaling baseline.
        wfull = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=device, generator=gen)
        sfull = (torch.rand(n, device=device, generator=gen) * 1e-3).to(torch.bfloat16)
        ofull = torch.empty((m, n), dtype=torch.bfloat16, device=device)
        fcopies = max(1, min(8, -(-POOL_MIN_BYTES // (n * k))))
        wl_full = [wfull] + [torch.randint(-127, 128, (n, k), dtype=torch.int8, device=device, generator=gen)
                             for _ in range(fcopies - 1)]

        def full_gemm():
            from qtts_b200.quant import kernels as qk

            for c in range(SHARD_CALLS):
                qk.w8_gemm(x, wl_full[c % fcopies], sfull, None, out=ofull)

        single_us = time_graph(full_gemm)
        del wl_full, wfull, sfull, ofull
        if fused_ok:
            # One checked call first: a failed exchange (bounded waits, recorded in the
            # device status) must not turn every timed call into a wait-limit expiry.
            nat.device_status(reset=True)
            fused[0](x)
            torch.cuda.synchronize()
            fused_ok = max_over_ranks(world, float(nat.device_status())) == 0.0
            if not fused_ok:
                fused_error = f"device status after the first fused call at K={k} N={n} M={m}"
        fused_us = time_graph(fused_calls) if fused_ok else None
        total_us = gemm_us + gather_us
        best_us = min(v for v in (gemm_gather_graph_us, fused_us) if v)
        res[f"K{k}_N{n}_M{m}"] = {
            "gemm_us": round(gemm_us, 3),
            "allgather_us": round(gather_us, 3),
            "gemm_allgather_us": round(total_us, 3),
            "gemm_allgather_graph_us": round(gemm_gather_graph_us, 3),
            "single_gpu_unsharded_us": round(single_us, 3),
            "sharded_efficiency": round(single_us / (world * best_us), 4),
            "fused_gemm_allgather_us": round(fused_us, 3) if fused_us else None,
            "fused_speedup": round(total_us / fused_us, 3) if fused_us else None,
            "agg_weight_gbs": round(n * k / (total_us * 1e-6) / 1e9, 1),
            "agg_weight_gbs_fused": round(n * k / (fused_us * 1e-6) / 1e9, 1) if fused_us else None,
            "agg_weight_gbs_gemm_only": round(n * k / (gemm_us * 1e-6) / 1e9, 1),
            "per_gpu_frac_of_hbm": round(rows * k / (gemm_us * 1e-6) / 1e9 / pk["hbm_gbs"], 4),
        }
        del ws, ss, lins, fused, x, block, gathered
        torch.cuda.empty_cache()
    # Parity of the gathered output at every rank against the unsharded GEMM.
    parity = {}
    for k, n, m in SHARD_PARITY_POINTS:
        parity[f"K{k}_N{n}_M{m}"] = round(sharded_parity(world, rank, device, seed, k, n, m), 6)
        torch.cuda.empty_cache()
    parity_ok = all(0 <= v <= 1e-2 for v in parity.values())
    return {
        "workload": "config 5: int8 W8A16 GEMM sharded along N over the ranks (ceil(N/g) rows each), bf16 "
        "outputs all-gathered over NCCL (gemm_allgather_us) or by the GEMM kernel itself over peer memory "
        "(fused_gemm_allgather_us); K in {2048,6144}, N in {12288,49152}, M in {1,8,64}",
        "scaling": "strong",
        "n_gpus": world,
        "allgather_timed": "allgather_us: eager loop, CUDA events; gemm_allgather_graph_us: GEMM + NCCL all-gather "
        "captured in one CUDA graph" if world > 1 else "single GPU: no exchange",
        "fused_error": fused_error,
        "sharded_parity_ok": parity_ok,
        "sharded_max_rel_err": parity,
        "sharded_efficiency": {key: v["sharded_efficiency"] for key, v in res.items() if key.startswith("K6144_N49152")},
        "per_point": res,
    }


class FusedMathFp32:
    """The math of the reference's int8 kernel (qtts/quant/kernels.py:114-135) in torch fp32:
    x times the exact int8 weight, fp32 accumulation, the per-channel scale after the K loop,
    then the cast. The parity check of config 4 (TF32 off)."""

    name = "fused_math_fp32"

    def apply(self, layer, x, bias):
        acc = torch.nn.functional.linear(x.float(), layer.int8_weight.float()) * layer.int8_scale.float()
        if bias is not None:
            acc = acc + bias.float()
        return acc.to(x.dtype)

    # The frame fuses its norms and SiLU·up into the int8 linears: the reference math
    # takes the same prologues (the library's RMSNorm, torch's SiLU·up, equal to the
    # library's), so only the GEMM arithmetic differs.
    def apply_rmsnorm(self, layer, x, norm_weight, eps, bias):
        from qtts_b200.quant import kernels as qk

        return self.apply(layer, qk.rms_norm(x, norm_weight, eps), bias)

    def apply_silu_mul(self, layer, gate_up, bias):
        gate, up = gate_up.chunk(2, dim=-1)
        return self.apply(layer, torch.nn.functional.silu(gate) * up, bias)


def talker_frames(seed: int, batch: int = 8) -> dict:
    """Config 4: frames/s of the random-init talker decode step + code predictor at batch 8 in
    one CUDA graph: all linears bf16 (cuBLAS), all linears int8 weight-only (this library),
    and int8 where calibration measures it faster (the reference's default); plus the codes
    of the all-int8 frame against the reference kernel's math in fp32 on the same weights."""
    from qtts_b200.config import QuantConfig
    from qtts_b200.decode_step import Block, Frame, timed_frames_per_s
    from qtts_b200.layers.linear import iter_linears
    from qtts_b200.quant import build_method, quantize_module

    frame = Frame(batch, seed=seed)
    fps_bf16, ms_bf16 = timed_frames_per_s(frame)
    bytes_bf16 = frame.frame_weight_bytes()
    frame.graph = None
    cfg = QuantConfig(method="int8_weight_only", targets=("talker", "code_predictor"), exclude_substrings=(),
                      calibrate=False)
    method = build_method(cfg)
    rep_t = quantize_module(frame.talker, method, cfg, "talker")
    rep_p = quantize_module(frame.predictor, method, cfg, "code_predictor")
    torch.cuda.empty_cache()
    fps_int8, ms_int8 = timed_frames_per_s(frame)
    codes = frame.codes.clone()
    # The same int8 frame with the code predictor's heads, argmax and next-embedding lookup
    # as separate ops instead of the library's fused head.
    from qtts_b200.decode_step import CodePredictor as _CP

    _CP.fuse_heads = False
    frame.graph = None
    try:
        fps_sep_heads, ms_sep_heads = timed_frames_per_s(frame)
    finally:
        _CP.fuse_heads = True
        frame.graph = None
    # The same int8 frame with the norms and SiLU·up as separate torch ops.
    Block.fuse_prologues = False
    frame.graph = None
    try:
        fps_unfused, ms_unfused = timed_frames_per_s(frame)
    finally:
        Block.fuse_prologues = True
        frame.graph = None
    # Same int8 weights through the reference kernel's math in fp32.
    layers = [layer for _, layer in iter_linears(frame.talker)] + [layer for _, layer in iter_linears(frame.predictor)]
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    ref_method = FusedMathFp32()
    for layer in layers:
        layer.quant_method = ref_method
    ref = frame.run().clone()
    torch.backends.cuda.matmul.allow_tf32 = tf32
    for layer in layers:
        layer.quant_method = method
    bytes_int8 = frame.frame_weight_bytes()
    del frame
    torch.cuda.empty_cache()
    # int8 only where calibration measures it faster than bf16 (--quant-calibrate, the default).
    frame = Frame(batch, seed=seed)
    cal = QuantConfig(method="int8_weight_only", targets=("talker", "code_predictor"), exclude_substrings=())
    cal_method = build_method(cal, calibration_batch=batch)
    cal_t = quantize_module(frame.talker, cal_method, cal, "talker")
    cal_p = quantize_module(frame.predictor, cal_method, cal, "code_predictor")
    torch.cuda.empty_cache()
    fps_cal, ms_cal = timed_frames_per_s(frame)
    del frame
    torch.cuda.empty_cache()
    return {
        "workload": "config 4: random-init talker decode step (28 layers, 512-token KV cache, masked codec head) "
        "+ code predictor (5 layers, 15 sequential codebook steps, 15 heads) at batch 8, one CUDA graph per frame; "
        "median of 5 windows of 20 replays",
        "frames_per_s_int8": round(fps_int8, 1),
        "frames_per_s_bf16": round(fps_bf16, 1),
        "frames_per_s_int8_separate_heads": round(fps_sep_heads, 1),
        "ms_per_step_int8_separate_heads": round(ms_sep_heads, 3),
        "frames_per_s_int8_torch_prologues": round(fps_unfused, 1),
        "ms_per_step_int8_torch_prologues": round(ms_unfused, 3),
        "speedup_vs_bf16": round(fps_int8 / fps_bf16, 3),
        "ms_per_step_int8": round(ms_int8, 3),
        "ms_per_step_bf16": round(ms_bf16, 3),
        "linear_weight_bytes_per_step": {"int8": bytes_int8, "bf16": bytes_bf16},
        "weight_gbs_int8": round(bytes_int8 / (ms_int8 * 1e-3) / 1e9, 1),
        "layers_int8": {"talker": rep_t.get("converted"), "code_predictor": rep_p.get("converted")},
        "frames_per_s_int8_calibrated": round(fps_cal, 1),
        "layers_int8_calibrated": {"talker": cal_t.get("converted"), "code_predictor": cal_p.get("converted"),
                                   "declined": (cal_t.get("declined") or 0) + (cal_p.get("declined") or 0)},
        "code0_match_vs_fused_math_fp32": float((codes[:, 0] == ref[:, 0]).float().mean().item()),
        "all_codes_match_vs_fused_math_fp32": float((codes == ref).float().mean().item()),
    }


def triton_sweep(points, xs, outs, pools, per_point, stream) -> str:
    """Time the reference's Triton ``w8_gemm`` (qtts/quant/kernels.py:89-177, installed
    unmodified under baseline/_ref) at every config-2 point: the same x, the same rotating
    weight pool and the same CUDA-graph form as the library's calls. Adds ``triton_us`` and
    ``speedup_vs_triton`` per point; returns "ok" or why the reference could not run."""
    try:
        from baseline import ref_frame as rf

        ref_gemm = rf.qtts().quant.kernels.w8_gemm
        for pt in points:
            x, out = xs[(pt.label, pt.m)], outs[(pt.label, pt.m)]
            qs, ss = pools[pt.label]
            check = ref_gemm(x, qs[0], ss[0])

            def tcalls(x=x, qs=qs, ss=ss):
                p = qs.shape[0]
                for c in range(CALLS_PER_GRAPH):
                    ref_gemm(x, qs[c % p], ss[c % p])

            us = graph_us_per_call(tcalls)
            d = per_point[pt.label][str(pt.m)]
            d["triton_us"] = round(us, 3)
            d["speedup_vs_triton"] = round(us / d["us"], 3)
            torch.cuda.synchronize()
            from qtts_b200.quant import kernels as qk

            mine = qk.w8_gemm(x, qs[0], ss[0])
            d["rel_err_vs_triton"] = float(((mine.float() - check.float()).abs().max()
                                            / check.float().abs().max().clamp_min(1e-30)).item())
        torch.cuda.empty_cache()
        return "ok"
    except Exception as exc:  # the comparison arm is optional; the library's numbers stand alone
        torch.cuda.synchronize()
        return f"unavailable: {type(exc).__name__}: {str(exc).splitlines()[0] if str(exc) else ''}"


def reference_model_frames(seed: int, batch: int = 8) -> dict:
    """Config 4 on the reference's own model (baseline/ref_frame.py): its Qwen3TTSTalker and
    CodePredictor, quantized by its apply_quantization (every linear, exclude_substrings=())
    and replayed through its TalkerDecodeGraphs / CodePredictorGraphs, one frame as its
    TalkerRunner.decode_step runs it (greedy). Arms: bf16; int8 on the reference's Triton
    kernel; int8 on this library (the one-file kernel swap), both uncalibrated on the same
    weights and calibrated (--quant-calibrate, each arm's kernel timed against F.linear);
    plus the greedy code-0 ids of one talker step, library against the reference's eager
    dequantize-then-matmul and Triton paths, with the top-1/top-2 logit margins."""
    import gc

    try:
        from baseline import ref_frame as rf

        rf.qtts()
    except Exception as exc:
        return {"unavailable": f"{type(exc).__name__}: {exc}"}
    out: dict = {"workload": "reference Qwen3TTSTalker + CodePredictor (baseline/_ref, unmodified) at batch 8, "
                 "512 prior tokens (key length bucketed to 768), its own CUDA graphs, greedy; frames/s = batch / "
                 "median frame time of 5 windows of 20 frames", "errors": {}}

    def release():
        gc.collect()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()

    def timed(key, talker, predictor):
        try:
            fr = rf.RefFrame(talker, predictor, batch, seed)
            fps, ms = fr.frames_per_s()
            out[f"frames_per_s_{key}"] = round(fps, 1)
            out[f"ms_per_frame_{key}"] = round(ms, 3)
            del fr
        except Exception as exc:
            out["errors"][key] = f"{type(exc).__name__}: {str(exc).splitlines()[0] if str(exc) else ''}"
        release()

    talker, predictor, _ = rf.build_models(batch=batch, quant=None, seed=seed)
    timed("ref_bf16", talker, predictor)
    del talker, predictor
    release()

    talker, predictor, rep = rf.build_models(batch=batch, quant="int8_weight_only", calibrate=False,
                                             kernels="library", seed=seed)
    out["layers_int8"] = {k: v.get("converted") for k, v in rep.items()}
    for kind, key in (("triton", "ref_triton"), ("library", "ref_model_with_library")):
        rf.set_kernels(kind)
        timed(key, talker, predictor)
    # code-0 parity on one talker step (same int8 buffers, three GEMMs)
    try:
        _, embeds = rf.initial_state(batch, seed)
        logits = {}
        for kind in ("library", "eager", "triton"):
            rf.set_kernels(kind)
            logits[kind] = rf.talker_step_logits(talker, embeds.clone()).float()
        top2 = logits["eager"].topk(2, dim=-1).values
        finite = torch.isfinite(logits["eager"])
        ids = {k: v.argmax(-1) for k, v in logits.items()}
        out["code0_library_vs_ref_eager"] = float((ids["library"] == ids["eager"]).float().mean().item())
        out["code0_library_vs_ref_triton"] = float((ids["library"] == ids["triton"]).float().mean().item())
        out["code0_top1_top2_margins"] = [round(v, 4) for v in (top2[:, 0] - top2[:, 1]).tolist()]
        out["logit_max_abs_diff_library_vs_eager"] = round((logits["library"] - logits["eager"])[finite].abs().max().item(), 5)
        out["logit_max_abs_diff_triton_vs_eager"] = round((logits["triton"] - logits["eager"])[finite].abs().max().item(), 5)
    except Exception as exc:
        out["errors"]["code0"] = f"{type(exc).__name__}: {str(exc).splitlines()[0] if str(exc) else ''}"
    rf.set_kernels("library")
    del talker, predictor
    release()

    for kind, key in (("triton", "ref_triton_calibrated"), ("library", "ref_model_with_library_calibrated")):
        try:
            talker, predictor, rep = rf.build_models(batch=batch, quant="int8_weight_only", calibrate=True,
                                                     kernels=kind, seed=seed)
            out[f"layers_int8_{key}"] = {k: {"converted": v.get("converted"), "declined": v.get("declined")}
                                         for k, v in rep.items()}
            timed(key, talker, predictor)
            del talker, predictor
        except Exception as exc:
            out["errors"][key] = f"{type(exc).__name__}: {str(exc).splitlines()[0] if str(exc) else ''}"
        release()
    rf.set_kernels("library")
    if "frames_per_s_ref_triton" in out and "frames_per_s_ref_model_with_library" in out:
        out["speedup_library_vs_triton"] = round(out["frames_per_s_ref_model_with_library"]
                                                 / out["frames_per_s_ref_triton"], 3)
    if not out["errors"]:
        del out["errors"]
    return out


def auto_kernel(m: int, n: int, k: int) -> str:
    """The kernel the library's automatic choice launches (asked of the library's planner)."""
    from qtts_b200 import _native as nat

    return nat.plan(m, n, k)["kernel"]


def run_gpu_arm(args) -> None:
    from qtts_b200 import _native as nat
    from qtts_b200.quant import kernels as qk

    world, rank, local = dist_init()
    device = torch.device("cuda", local)
    ok, reason = qk.kernel_available()
    if not ok:
        raise RuntimeError(reason)
    pools = build_pools(device, seed=args.seed)
    gen = torch.Generator(device=device)
    gen.manual_seed(args.seed + 1)

    points: list[Point] = []
    xs, outs, xs_host, outs_host = {}, {}, {}, {}
    for m in ROWS:
        for label, n, k in SHAPES:
            pt = Point(label, n, k, m)
            x = torch.randn((m, k), generator=gen, device=device).to(torch.bfloat16)
            out = torch.empty((m, n), dtype=torch.bfloat16, device=device)
            xs[(label, m)], outs[(label, m)] = x, out
            xs_host[(label, m)] = x.cpu().pin_memory()
            outs_host[(label, m)] = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
            qs, ss = pools[label]
            variant = nat.VARIANT_AUTO if args.variant is None else int(args.variant, 0)

            def calls(x=x, out=out, qs=qs, ss=ss, variant=variant):
                p = qs.shape[0]
                for c in range(CALLS_PER_GRAPH):
                    qk.w8_gemm(x, qs[c % p], ss[c % p], None, out=out, variant=variant)

            pt.graph = capture(calls)
            points.append(pt)

    bytes_per_step = sum(pt.bytes for pt in points) * CALLS_PER_GRAPH * REPLAYS_PER_POINT
    launches_per_step = len(points) * CALLS_PER_GRAPH * REPLAYS_PER_POINT
    stream = torch.cuda.current_stream()

    def step(events=None):
        for i, pt in enumerate(points):
            for _ in range(REPLAYS_PER_POINT):
                pt.graph.replay()
            if events is not None:
                events[i].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)

    sampler = ClockSampler(local, Path(os.environ["QTTS_BENCH_CLOCKS_LOG"]) if "QTTS_BENCH_CLOCKS_LOG" in os.environ
                           else None)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    point_events = [[torch.cuda.Event(enable_timing=True) for _ in points] for _ in range(args.steps)]
    start.record(stream)
    for s in range(args.steps):
        step(point_events[s])
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(end)
    elapsed_ms_max = max_over_ranks(world, elapsed_ms)

    # per-point device time, averaged over steps
    per_point_ms = [0.0] * len(points)
    for s in range(args.steps):
        prev = start if s == 0 else point_events[s - 1][-1]
        for i, ev in enumerate(point_events[s]):
            per_point_ms[i] += (prev.elapsed_time(ev)) / args.steps
            prev = ev

    value = bytes_per_step * args.steps * world / (elapsed_ms_max * 1e-3) / 1e9
    pk = peaks()
    # Roofline of the dominant kernel: its algorithmic bytes per launch over
    # its average launch duration, from the per-point events of the timed
    # region (every call of a point launches the same kernel).
    by_kernel: dict = {}
    for pt, ms in zip(points, per_point_ms):
        kname = auto_kernel(pt.m, pt.n, pt.k) if args.variant is None else f"variant {args.variant}"
        kb, kt = by_kernel.get(kname, (0.0, 0.0))
        by_kernel[kname] = (kb + pt.bytes * CALLS_PER_GRAPH * REPLAYS_PER_POINT, kt + ms)
    dom_kernel = max(by_kernel, key=lambda kk: by_kernel[kk][1])
    dom_bytes, dom_ms = by_kernel[dom_kernel]
    dom_gbs = dom_bytes / (dom_ms * 1e-3) / 1e9
    calls_per_point = CALLS_PER_GRAPH * REPLAYS_PER_POINT
    per_point = {}
    for pt, ms in zip(points, per_point_ms):
        us = ms * 1e3 / calls_per_point
        per_point.setdefault(pt.label, {})[str(pt.m)] = {
            "us": round(us, 3),
            "gbs": round(pt.bytes / (us * 1e-6) / 1e9, 1),
        }

    # ---- cuBLAS bf16 comparison (outside the timed region)
    if args.bf16_compare:
        bf16_pools = {}
        for label, n, k in SHAPES:
            qs, ss = pools[label]
            p = pool_size(n, k)
            bf16_pools[label] = [(qs[i].to(torch.bfloat16) * ss[i][:, None]) for i in range(p)]
        for pt in points:
            x, out = xs[(pt.label, pt.m)], outs[(pt.label, pt.m)]
            wl = bf16_pools[pt.label]

            def bcalls(x=x, wl=wl):
                for c in range(CALLS_PER_GRAPH):
                    torch.nn.functional.linear(x, wl[c % len(wl)])

            g = capture(bcalls)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g.replay()
            e0.record(stream)
            for _ in range(3):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (3 * CALLS_PER_GRAPH)
            d = per_point[pt.label][str(pt.m)]
            d["bf16_us"] = round(us, 3)
            d["speedup_vs_bf16"] = round(us / d["us"], 3)
            del g
        del bf16_pools
        torch.cuda.empty_cache()

    # ---- the reference's own Triton kernel on the same points (outside the timed region)
    triton_status = None
    if args.triton_compare:
        triton_status = triton_sweep(points, xs, outs, pools, per_point, stream)

    torch.cuda.synchronize()
    status_sweep = nat.device_status()  # before the sections (the sharded one resets the word)

    # ---- config 3 (fp8) and config 5 (N-sharded GEMM + all-gather), outside the timed region
    fp8 = fp8_sweep(device, args.seed) if args.fp8 and rank == 0 else None
    fp8w = fp8w_sweep(device, args.seed) if args.fp8w and rank == 0 else None
    w8a8 = w8a8_sweep(device, args.seed) if args.w8a8 and rank == 0 else None
    prologue = prologue_sweep(device, args.seed) if args.prologue and rank == 0 else None
    heads = grouped_heads(device, args.seed) if args.heads and rank == 0 else None
    barrier(world)
    sharded = sharded_sweep(world, rank, device, args.seed) if args.sharded else None
    talker = talker_frames(args.seed) if args.talker and rank == 0 else None
    if talker is not None and args.ref_model:
        talker["reference_model"] = reference_model_frames(args.seed)
    barrier(world)

    # ---- end to end through the public API with host buffers: every call copies its x in
    # from pinned host memory and its output back out (both copies captured with the call).
    calls_per_step = CALLS_PER_GRAPH * REPLAYS_PER_POINT
    h2d = sum(pt.m * pt.k * 2 for pt in points) * calls_per_step
    d2h = sum(pt.m * pt.n * 2 for pt in points) * calls_per_step
    variant = nat.VARIANT_AUTO if args.variant is None else int(args.variant, 0)
    for pt in points:
        key = (pt.label, pt.m)
        qs, ss = pools[pt.label]

        def e2e_calls(x=xs[key], out=outs[key], xh=xs_host[key], oh=outs_host[key], qs=qs, ss=ss):
            p = qs.shape[0]
            for c in range(CALLS_PER_GRAPH):
                x.copy_(xh, non_blocking=True)
                qk.w8_gemm(x, qs[c % p], ss[c % p], None, out=out, variant=variant)
                oh.copy_(out, non_blocking=True)

        pt.graph = None
        pt.e2e_graph = capture(e2e_calls)

    def e2e_step():
        for pt in points:
            for _ in range(REPLAYS_PER_POINT):
                pt.e2e_graph.replay()

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(world, e0.elapsed_time(e1))
    e2e_value = bytes_per_step * args.steps * world / (e2e_ms * 1e-3) / 1e9

    status = status_sweep or nat.device_status()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_port_sample(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms_max / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": "config-2 talker linear sweep: qkv 4096x2048, o_proj 2048x2048, gate_up 12288x2048, "
                "down 2048x6144 at M in {1,2,4,8,16,32,64}; 2016 calls per point per step",
                "global_batch": None,
                "l2": "weights rotate through >= 256 MB per shape (> 2x L2); every call reads its weight from HBM",
                "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                "variant": args.variant or "auto",
            },
            "roofline": {
                "bound": "hbm",
                "kernel": dom_kernel,
                "achieved": round(dom_gbs, 1),
                "peak": pk["hbm_gbs"],
                "unit": "GB/s",
                "frac": round(dom_gbs / pk["hbm_gbs"], 4),
                "peak_source": pk["source"],
                "share_of_step": round(dom_ms / sum(per_point_ms), 3),
                "traffic": NCU_TRAFFIC["bytes_per_launch"],
                "traffic_case": NCU_TRAFFIC,
                "by_kernel_gbs": {kk: round(b / (t * 1e-3) / 1e9, 1) for kk, (b, t) in by_kernel.items()},
            },
            "cpu_baseline": cpu,
            "e2e": {
                "value": round(e2e_value, 1),
                "unit": "GB/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
            },
            "clocks": clocks,
            "gpu_launches": launches_per_step * args.steps,
            "device_status": status,
            "triton_compare": triton_status,
            "per_point": per_point,
            "fp8": fp8,
            "fp8_weight_only": fp8w,
            "int8_w8a8": w8a8,
            "fused_prologues": prologue,
            "grouped_heads": heads,
            "sharded": sharded,
            "talker": talker,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        for pt in points:
            pt.graph = None
            pt.e2e_graph = None
        dist.destroy_process_group()


def run_single(spec: str, calls: int = 3) -> None:
    """One (shape, M) point, `calls` launches with an L2 flush before each:
    a small case for `ncu` captures. spec = "<shape>:<M>[:<variant>]" (W8A16),
    "fp8:<shape>:<M>" (activation quantization + fp8 GEMM), "fp8w:<shape>:<M>"
    (fp8 weight-only), "rms:<shape>:<M>" / "silu:<shape>:<M>" (W8A16 with its
    RMSNorm / SiLU·up prologue, qtts_w8a16_gemm_prologue), "frame" (one eager
    config-4 frame inside a CUDA profiler range) or "refframe:<bf16|triton|library>" (one
    frame of the reference's own model and CUDA graphs, int8 on the named kernel, inside a
    CUDA profiler range after three warm frames)."""
    from qtts_b200.quant import kernels as qk

    parts = spec.split(":")
    if parts[0] == "refframe":
        from baseline import ref_frame as rf

        arm = parts[1] if len(parts) > 1 else "library"
        if arm not in ("bf16", "triton", "library"):
            raise ValueError(f"refframe arm must be bf16, triton or library, not {arm!r}")
        torch.cuda.set_device(0)
        talker, predictor, _ = rf.build_models(batch=8, quant=None if arm == "bf16" else "int8_weight_only",
                                               seed=0, kernels="triton" if arm == "triton" else "library")
        fr = rf.RefFrame(talker, predictor, 8, 0)
        for _ in range(3):
            fr.step()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        fr.step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"single": spec, "ok": True}))
        return
    if parts[0] == "frame":
        # One eager config-4 frame (batch 8, all linears int8 with the fused prologues), with
        # the CUDA profiler range opened around it only (ncu --profile-from-start off).
        from qtts_b200.config import QuantConfig
        from qtts_b200.decode_step import Frame
        from qtts_b200.quant import build_method, quantize_module

        torch.cuda.set_device(0)
        frame = Frame(8, seed=0)
        cfg = QuantConfig(method="int8_weight_only", targets=("talker", "code_predictor"), exclude_substrings=(),
                          calibrate=False)
        method = build_method(cfg)
        quantize_module(frame.talker, method, cfg, "talker")
        quantize_module(frame.predictor, method, cfg, "code_predictor")
        with torch.no_grad():
            frame.run()
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            frame.run()
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
        print(json.dumps({"single": spec, "ok": True}))
        return
    if parts[0] in ("rms", "silu"):
        label, m = parts[1], int(parts[2])
        n, k = {lab: (n_, k_) for lab, n_, k_ in SHAPES}[label]
        torch.cuda.set_device(0)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(0)
        q, s_ = qk.quantize_int8_rows(torch.randn((n, k), generator=gen, device="cuda") * 0.02)
        s_ = s_.to(torch.bfloat16)
        width = k if parts[0] == "rms" else 2 * k
        x = torch.randn((m, width), generator=gen, device="cuda").to(torch.bfloat16)
        nw = torch.ones(k, dtype=torch.bfloat16, device="cuda")
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        for _ in range(calls):
            flush.zero_()
            if parts[0] == "rms":
                qk.w8_gemm_rmsnorm(x, nw, 1e-6, q, s_)
            else:
                qk.w8_gemm_silu_mul(x, q, s_)
        torch.cuda.synchronize()
        print(json.dumps({"single": spec, "ok": True}))
        return
    if parts[0] == "fp8w":
        label, m = parts[1], int(parts[2])
        n, k = {lab: (n_, k_) for lab, n_, k_ in SHAPES}[label]
        torch.cuda.set_device(0)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(0)
        w = torch.randn((n, k), generator=gen, device="cuda") * 0.02
        wq, ws = qk.quantize_fp8_rows(w)
        x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        for _ in range(calls):
            flush.zero_()
            qk.fp8w_gemm(x, wq, ws)
        torch.cuda.synchronize()
        print(json.dumps({"single": spec, "ok": True}))
        return
    if parts[0] == "fp8":
        label, m = parts[1], int(parts[2])
        n, k = {lab: (n_, k_) for lab, n_, k_ in SHAPES}[label]
        torch.cuda.set_device(0)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(0)
        w = torch.randn((n, k), generator=gen, device="cuda") * 0.02
        wq, ws = qk.quantize_fp8_rows(w)
        x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        for _ in range(calls):
            flush.zero_()
            xq, sx = qk.fp8_quant_rows(x)
            qk.fp8_scaled_mm(xq, sx, wq, ws, None, torch.bfloat16)
        torch.cuda.synchronize()
        print(json.dumps({"single": spec, "ok": True}))
        return
    label, m = parts[0], int(parts[1])
    variant = int(parts[2], 0) if len(parts) > 2 else 0
    n, k = {lab: (n_, k_) for lab, n_, k_ in SHAPES}[label]
    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    w = torch.randn((n, k), generator=gen, device="cuda") * 0.02
    q, s = qk.quantize_int8_rows(w)
    s = s.to(torch.bfloat16)
    x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(calls):
        flush.zero_()
        qk.w8_gemm(x, q, s, variant=variant)
    torch.cuda.synchronize()
    print(json.dumps({"single": spec, "ok": True}))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--variant", default=None, help="force a kernel variant (e.g. 0x104); default: library choice")
    ap.add_argument("--no-bf16-compare", dest="bf16_compare", action="store_false")
    ap.add_argument("--no-fp8", dest="fp8", action="store_false", help="skip the config-3 fp8 sweep")
    ap.add_argument("--no-fp8w", dest="fp8w", action="store_false", help="skip the fp8 weight-only sweep")
    ap.add_argument("--no-w8a8", dest="w8a8", action="store_false", help="skip the int8 W8A8 sweep")
    ap.add_argument("--no-prologue", dest="prologue", action="store_false",
                    help="skip the fused RMSNorm / SiLU·up sweep")
    ap.add_argument("--no-heads", dest="heads", action="store_false",
                    help="skip the grouped 15-codebook-head measurement")
    ap.add_argument("--no-talker", dest="talker", action="store_false",
                    help="skip the config-4 talker + code predictor frames/s measurement")
    ap.add_argument("--no-sharded", dest="sharded", action="store_false",
                    help="skip the config-5 N-sharded GEMM + all-gather sweep")
    ap.add_argument("--no-triton-compare", dest="triton_compare", action="store_false",
                    help="skip timing the reference's Triton w8_gemm per point")
    ap.add_argument("--no-ref-model", dest="ref_model", action="store_false",
                    help="skip the config-4 frame on the reference's own model")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--replays", type=int, default=REPLAYS_PER_POINT,
                    help="graph replays per point per step (224 calls each); 9 gives the reference's 2016 calls")
    ap.add_argument("--single", default=None,
                    help="profile case: run one point '<shape>:<M>[:<variant>]' 3 times and exit")
    args = ap.parse_args(argv)
    globals()["REPLAYS_PER_POINT"] = args.replays
    if args.single:
        run_single(args.single)
        return 0
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_gpu_arm(args)
    return 0


if __name__ == "__main__":
    sys.exit(main())
