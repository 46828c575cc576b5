"""N-sharded W8A16 linear over a world_size-2 gloo group on CPU.

The local products come from the CPU oracle (injected, as the test's own
checker); what is tested is the host side of the multi-GPU path: which rows
each rank owns, the rank-major all-gather and the reassembly into [M, N],
including an N that does not divide by the world size.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from qtts_b200.sharded import ShardedW8Linear, shard_rows, shard_width


def test_shard_rows_cover_every_row_once():
    for n in (1, 7, 16, 12288, 12289, 49152):
        for world in (1, 2, 3, 4, 8):
            got = [shard_rows(n, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n
            for (a0, a1), (b0, b1) in zip(got, got[1:]):
                assert a1 == b0 and a0 <= a1
            assert all(b - a <= shard_width(n, world) for a, b in got)
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_gemm(x, w, s, b):
    out = oracle.w8a16_reference(x.float().numpy(), w.numpy(), s.float().numpy(),
                                 None if b is None else b.float().numpy())
    return torch.from_numpy(out).to(x.dtype)


def _worker(rank: int, world: int, port: int, n: int, k: int, m: int, q: np.ndarray, s: np.ndarray,
            x: np.ndarray, queue) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        start, stop = shard_rows(n, world, rank)
        lin = ShardedW8Linear(torch.from_numpy(q[start:stop]), torch.from_numpy(s[start:stop]), n, gemm=_cpu_gemm)
        y = lin(torch.from_numpy(x).to(torch.float32))
        if rank == 0:
            queue.put(y.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [64, 77])
def test_gloo_world2_matches_unsharded(n):
    k, m, world = 96, 3, 2
    g = torch.Generator().manual_seed(80)
    w = torch.randn(n, k, generator=g) * 0.02
    q, s = oracle.quantize_weight_per_channel(w.numpy())
    x = torch.randn(m, k, generator=g).numpy()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, k, m, q, s, x, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = queue.get(timeout=60)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = oracle.w8a16_reference(x, q, s)
    assert got.shape == (m, n)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


class _Addr:
    """A peer mapping as the fused class sees it: only its device address."""

    def __init__(self, ptr: int) -> None:
        self.ptr = ptr

    def data_ptr(self) -> int:
        return self.ptr


def _fused_worker(rank: int, world: int, port: int, n: int, k: int, m: int, q: np.ndarray, s: np.ndarray,
                  x: np.ndarray, queue) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qtts_b200.sharded import FusedAllGatherW8Linear

        def exchange(t, group):
            addrs = [None] * world
            dist.all_gather_object(addrs, t.data_ptr(), group=group)
            return [t if r == rank else _Addr(a) for r, a in enumerate(addrs)]

        holder: dict = {}

        def launch(x, w, s, b, *, peer_out, ldo, col_offset, peer_signal, sync, rank, world):
            # Stand-in for the kernel: this rank's block goes to every rank's gathered
            # buffer at its column offset (here by an object all-gather).
            blocks = [None] * world
            dist.all_gather_object(blocks, (col_offset, _cpu_gemm(x, w, s, b).numpy()))
            lin = holder["lin"]
            for off, blk in blocks:
                lin.gathered[: blk.shape[0], off: off + blk.shape[1]] = torch.from_numpy(blk)
            holder["args"] = (ldo, col_offset, peer_out.tolist(), peer_signal.tolist(), rank, world)

        start, stop = shard_rows(n, world, rank)
        lin = FusedAllGatherW8Linear(torch.from_numpy(q[start:stop]), torch.from_numpy(s[start:stop]), n,
                                     max_rows=8, dtype=torch.float32, exchange=exchange, launch=launch)
        holder["lin"] = lin
        y = lin(torch.from_numpy(x).to(torch.float32))
        queue.put((rank, y.numpy(), holder["args"], lin.gathered.data_ptr(), lin.signal.data_ptr()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [64, 77])
def test_gloo_world2_fused_allgather_layout(n):
    """Host side of the fused GEMM + all-gather: column offsets, the gathered row
    stride, the peer tables in rank order, and the [M, N] view of the result."""
    k, m, world = 96, 3, 2
    g = torch.Generator().manual_seed(81)
    w = torch.randn(n, k, generator=g) * 0.02
    q, s = oracle.quantize_weight_per_channel(w.numpy())
    x = torch.randn(m, k, generator=g).numpy()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, n, k, m, q, s, x, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted((queue.get(timeout=60) for _ in range(world)), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = oracle.w8a16_reference(x, q, s)
    shard = shard_width(n, world)
    out_ptrs = [r[3] for r in results]
    sig_ptrs = [r[4] for r in results]
    for rank, y, (ldo, col_offset, peer_out, peer_sig, r_rank, r_world), _, _ in results:
        assert y.shape == (m, n)
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)
        assert (ldo, col_offset, r_rank, r_world) == (world * shard, rank * shard, rank, world)
        assert peer_out == out_ptrs and peer_sig == sig_ptrs
