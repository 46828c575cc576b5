"""Per-shape measurement: is the quantized GEMM faster here, and with which kernel?

Same method as qtts/quant/calibrate.py: time both GEMMs inside a captured CUDA
graph (``inner`` calls per graph, ``iters`` replays; calibrate.py:40-63) and
quantize a shape only when ``t_quantized * margin < t_reference``
(calibrate.py:77-114). A capture failure declines instead of failing
(calibrate.py:97-103). Verdicts are cached per key.

What this module adds is the kernel-variant choice: the library has several
kernels for one shape (split-K factors of the skinny kernel, the SIMT
fallback), and which is fastest depends on the shape and the batch rows. The
cache therefore maps a key to ``(verdict, variant)``: ``choose_variant`` times
each candidate once, and ``worth_quantizing`` compares the winner against the
unquantized GEMM.
"""

from __future__ import annotations

import time
from typing import Callable

import torch

from ..utils import get_logger

logger = get_logger("quant.calibrate")

_CACHE: dict[tuple, bool] = {}
_VARIANTS: dict[tuple, int] = {}


def graph_time(fn: Callable[[], object], inner: int = 10, iters: int = 50) -> float:
    """Seconds per call of ``fn``, measured from a captured graph."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(inner):
            fn()
    torch.cuda.synchronize()
    started = time.perf_counter()
    for _ in range(iters):
        graph.replay()
    torch.cuda.synchronize()
    elapsed = (time.perf_counter() - started) / (iters * inner)
    del graph
    return elapsed


def eager_time(fn: Callable[[], object], iters: int = 200) -> float:
    for _ in range(20):
        fn()
    torch.cuda.synchronize()
    started = time.perf_counter()
    for _ in range(iters):
        fn()
    torch.cuda.synchronize()
    return (time.perf_counter() - started) / iters


def choose_variant(candidates: dict[int, Callable[[], object]], *, key: tuple, use_graph: bool = True) -> int:
    """The fastest variant among ``candidates`` (variant -> call), cached by ``key``.

    A candidate that raises (not applicable to the shape, capture failure) is
    skipped. Returns 0 (the library's own choice) when none could be timed.
    """
    if key in _VARIANTS:
        return _VARIANTS[key]
    timer = graph_time if use_graph else eager_time
    best, best_t = 0, float("inf")
    for variant, call in candidates.items():
        try:
            t = timer(call)
        except Exception as exc:  # not applicable here; try the next one
            logger.debug("variant %#x failed for %s: %s", variant, key, exc)
            continue
        if t < best_t:
            best, best_t = variant, t
    _VARIANTS[key] = best
    logger.debug("%s: variant %#x at %.2f us", key, best, best_t * 1e6)
    return best


def worth_quantizing(
    quantized_call: Callable[[], object],
    reference_call: Callable[[], object],
    *,
    key: tuple,
    margin: float = 1.05,
    use_graph: bool = True,
) -> bool:
    """Whether ``quantized_call`` beats ``reference_call`` by ``margin``."""
    if key in _CACHE:
        return _CACHE[key]
    timer = graph_time if use_graph else eager_time
    try:
        reference = timer(reference_call)
        quantized = timer(quantized_call)
    except Exception as exc:
        # Capture can fail for reasons unrelated to the layer; declining to
        # quantize is the safe answer.
        logger.warning("calibration failed for %s (%s); leaving it unquantized", key, exc)
        _CACHE[key] = False
        return False
    verdict = quantized * margin < reference
    _CACHE[key] = verdict
    logger.debug(
        "%s: reference %.1f us, quantized %.1f us (%.2fx) -> %s",
        key,
        reference * 1e6,
        quantized * 1e6,
        reference / quantized,
        "quantize" if verdict else "keep",
    )
    return verdict


def lookup_variant(key: tuple) -> int | None:
    return _VARIANTS.get(key)


def clear_cache() -> None:
    _CACHE.clear()
    _VARIANTS.clear()
