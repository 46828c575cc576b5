"""N-sharded W8A16 GEMM fused with the all-gather of its output (qtts_w8a16_gemm_allgather).

On one GPU the world is one rank: the kernel stores into its own gathered
buffer and signals itself, which exercises the epilogue's peer-store path,
the per-call epoch kept on the device and the two flag phases without any
wait on another kernel. With two GPUs visible, two ranks (one process per GPU,
NCCL for setup only, NVLS off) map each other's buffers through CUDA IPC and
the gathered output is compared with the oracle and with the NCCL all-gather
form. Tolerance as for W8A16: within 1e-2 of max|ref| and every output within
one bf16 rounding (+1e-3 max|ref|) of the float64 oracle.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import oracle
from conftest import require_b200
from qtts_b200 import _native as nat
from qtts_b200.quant import kernels as qk
from qtts_b200.sharded import FusedAllGatherW8Linear, shard_rows

pytestmark = pytest.mark.gpu


def case(n, k, m, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    q, s = oracle.quantize_weight_per_channel(w.numpy())
    s_bf16 = torch.from_numpy(s).to(torch.bfloat16)
    return x, q, s_bf16


def reference(x, q, s_bf16):
    return oracle.w8a16_reference(x.float().numpy(), q, s_bf16.float().numpy())


def check(out, ref, what):
    out = out.float().cpu().numpy().astype(np.float64)
    err = oracle.rel_err(out, ref)
    assert err <= 1e-2, f"{what}: rel err {err:.3e}"
    bad = np.abs(out - ref) > np.abs(ref) * 2.0**-8 + 1e-3 * np.abs(ref).max()
    assert not bad.any(), f"{what}: {bad.sum()} elements beyond one bf16 rounding"


@pytest.fixture(scope="module")
def _device():
    require_b200()
    nat.device_status(reset=True)
    yield
    torch.cuda.synchronize()
    assert nat.device_status() == 0, "a kernel recorded a device-side failure"


@pytest.mark.parametrize("n,k,m", [(4096, 2048, 1), (12288, 2048, 8), (2048, 6144, 16), (1536, 2048, 64),
                                   (6144, 2048, 33), (80, 272, 3)])
def test_world1_matches_oracle(_device, n, k, m):
    x, q, s = case(n, k, m, seed=100)
    lin = FusedAllGatherW8Linear(torch.from_numpy(q).cuda(), s.cuda(), n, max_rows=64)
    for call in range(3):
        xc = x if call == 0 else torch.randn(m, k, generator=torch.Generator().manual_seed(101 + call)).to(x.dtype)
        out = lin(xc.cuda())
        assert out.shape == (m, n)
        check(out, reference(xc, q, s), f"N={n} K={k} M={m} call {call}")
    torch.cuda.synchronize()
    # Three calls: epoch 3 recorded, ready and done slots of the one rank at 3.
    assert lin.sync.tolist() == [0, 3]
    assert lin.signal.tolist() == [3, 3]


@pytest.mark.parametrize("variant", ["skinny2", "skinny8", "umma1", "umma4"])
def test_world1_forced_variants(_device, variant):
    n, k, m = 2048, 2048, 8 if variant.startswith("skinny") else 40
    x, q, s = case(n, k, m, seed=102)
    v = nat.variant_skinny(int(variant[-1])) if variant.startswith("skinny") else nat.variant_umma(int(variant[-1]))
    lin = FusedAllGatherW8Linear(torch.from_numpy(q).cuda(), s.cuda(), n, max_rows=64)
    qk.w8_gemm_allgather(x.cuda(), lin.weight, lin.scale, None, peer_out=lin.peer_out, ldo=lin.ldo, col_offset=0,
                         peer_signal=lin.peer_sig, sync=lin.sync, rank=0, world=1, variant=v)
    check(lin.gathered[:m, :n], reference(x, q, s), variant)


def test_world1_graph_replays(_device):
    n, k, m = 4096, 2048, 4
    x, q, s = case(n, k, m, seed=103)
    lin = FusedAllGatherW8Linear(torch.from_numpy(q).cuda(), s.cuda(), n, max_rows=8)
    xs = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        lin(xs)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = lin(xs)
    for r in range(3):
        xn = torch.randn(m, k, generator=torch.Generator().manual_seed(104 + r)).to(torch.bfloat16)
        xs.copy_(xn.cuda())
        graph.replay()
        torch.cuda.synchronize()
        check(out, reference(xn, q, s), f"replay {r}")
    # the warm-up call and three replays (capture records the launch without running it)
    assert lin.sync.tolist()[1] == 4


def test_rejects_what_it_cannot_fuse(_device):
    n, k, m = 256, 256, 2
    x, q, s = case(n, k, m, seed=105)
    lin = FusedAllGatherW8Linear(torch.from_numpy(q).cuda(), s.cuda(), n, max_rows=8)
    kw = dict(peer_out=lin.peer_out, ldo=lin.ldo, col_offset=0, peer_signal=lin.peer_sig, sync=lin.sync, rank=0,
              world=1)
    with pytest.raises(RuntimeError, match="inapplicable kernel variant"):
        qk.w8_gemm_allgather(x.cuda(), lin.weight, lin.scale, None, variant=nat.variant_stream(0), **kw)
    with pytest.raises(RuntimeError):
        qk.w8_gemm_allgather(x.cuda(), lin.weight, lin.scale, None, **{**kw, "col_offset": 1})  # past ldo
    with pytest.raises(RuntimeError):
        qk.w8_gemm_allgather(x.cuda(), lin.weight, lin.scale, None, **{**kw, "rank": 1})  # outside the world
    with pytest.raises(ValueError):
        lin(torch.zeros(9, k, dtype=torch.bfloat16, device="cuda"))  # beyond max_rows
    torch.cuda.synchronize()
    assert lin.sync.tolist() == [0, 0]  # nothing was launched


# ---------------------------------------------------------------------------- two ranks


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _two_rank_worker(rank, world, port, points, queue):
    import torch.distributed as dist

    from qtts_b200.sharded import ShardedW8Linear

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    failures = []
    try:
        nat.device_status(reset=True)
        for n, k, m, x, q, s in points:
            start, stop = shard_rows(n, world, rank)
            w_dev = torch.from_numpy(q[start:stop]).cuda()
            s_dev = s[start:stop].cuda()
            fused = FusedAllGatherW8Linear(w_dev, s_dev, n, max_rows=64)
            nccl = ShardedW8Linear(w_dev, s_dev, n)
            ref = reference(x, q, s)
            for call in range(3):
                got = fused(x.cuda())
                want = nccl(x.cuda())
                torch.cuda.synchronize()
                try:
                    check(got, ref, f"rank {rank} N={n} M={m} call {call} (fused)")
                    check(want, ref, f"rank {rank} N={n} M={m} call {call} (NCCL all-gather)")
                except AssertionError as exc:
                    failures.append(str(exc))
            del fused
            dist.barrier()
        if nat.device_status() != 0:
            failures.append(f"rank {rank}: device status {nat.device_status()}")
    except Exception as exc:  # reported to the parent
        failures.append(f"rank {rank}: {exc!r}")
    finally:
        queue.put((rank, failures))
        dist.destroy_process_group()


def test_two_ranks_over_peer_memory():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    require_b200()
    import torch.multiprocessing as mp

    points = []
    for n, k, m, seed in [(12288, 2048, 1, 110), (4096, 6144, 8, 111), (12288, 2048, 12, 114), (12288, 2048, 64, 112),
                          (77, 96, 3, 113)]:
        x, q, s = case(n, k, m, seed)
        points.append((n, k, m, x, q, s))
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, points, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    problems = [f for _, fs in results for f in fs]
    assert not problems, "\n".join(problems)
    assert all(p.exitcode == 0 for p in procs)
