"""Timed CPU baseline: the reference's eager dequantize-then-matmul on host cores.

TEST/MEASUREMENT INFRASTRUCTURE ONLY -- used by bench.py's CPU-baseline leg and
its ``--impl reference`` arm, never by the library.

The reference's only CPU-runnable form of the path is the eager expression of
examples/kernels/tune_w8_gemm.py:73-79 (the "naive w8" column):
``F.linear(x, q.to(bf16) * scale[:, None])``, run here with torch on the CPU
with every host thread. Weights are quantized with the oracle's restatement of
qtts/quant/int8.py:45-56 and the scale is stored in bf16 as
Int8WeightOnlyMethod does (int8.py:105).
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch
import torch.nn.functional as F

from .qtts_ref import quantize_weight_per_channel


def use_all_threads() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def eager_dequant_linear(x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """tune_w8_gemm.py:73-79: dequantize into memory, then a bf16 GEMM."""
    return F.linear(x, q.to(x.dtype) * scale[:, None])


def algo_bytes(n: int, k: int, m: int) -> int:
    return n * k + 2 * n + 2 * m * k + 2 * m * n


class SweepWork:
    """One call per (shape, M) point of the config-2 sweep, on the CPU."""

    def __init__(self, shapes, rows, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        self.weights = {}
        for label, n, k in shapes:
            w = (torch.randn(n, k, generator=g) * 0.02).numpy()
            q, s = quantize_weight_per_channel(w)
            self.weights[label] = (torch.from_numpy(q), torch.from_numpy(s).to(torch.bfloat16))
        self.points = []
        for m in rows:
            for label, n, k in shapes:
                x = torch.randn(m, k, generator=g).to(torch.bfloat16)
                self.points.append((label, n, k, m, x))
        self.bytes_per_step = sum(algo_bytes(n, k, m) for _, n, k, m, _ in self.points)

    def step(self) -> None:
        for label, _n, _k, _m, x in self.points:
            q, s = self.weights[label]
            eager_dequant_linear(x, q, s)


def time_sweep(shapes, rows, budget_s: float = 15.0, seed: int = 0) -> dict:
    """Run whole sweeps for about ``budget_s`` seconds; GB/s of algorithmic bytes."""
    threads = use_all_threads()
    work = SweepWork(shapes, rows, seed=seed)
    work.step()  # warm-up
    steps = 0
    t0 = time.perf_counter()
    while True:
        work.step()
        steps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    elapsed = time.perf_counter() - t0
    return {
        "value": round(work.bytes_per_step * steps / elapsed / 1e9, 3),
        "unit": "GB/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{steps} sweep(s) of one eager F.linear(x, q.to(bf16)*scale) per (shape, M) point "
        f"({len(work.points)} points), {elapsed:.1f} s",
        "ms_per_call_mean": round(elapsed / (steps * len(work.points)) * 1e3, 3),
    }


if __name__ == "__main__":  # pragma: no cover
    print(time_sweep([("gate_up", 12288, 2048)], (1,), budget_s=3.0))
    _ = np.zeros(1)
