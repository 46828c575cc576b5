"""Bounded device-side waits run out into QTTS_ERR_TIMEOUT instead of hanging.

The fused GEMM + all-gather (csrc/allgather.cuh) waits for every rank's "ready"
flag before its first output store and for every rank's "done" flag at the end.
Here one GPU calls it as rank 0 of a world of 2 whose rank 1 is a fake: its
gathered buffer and signal pad are plain local tensors that nothing ever
signals. With the wait limit at 1 ms the call must return, record
QTTS_ERR_TIMEOUT in the device status word, store no output anywhere (the
store gate failed), keep every cluster barrier of the split-K and tcgen05
kernels (no CTA is left waiting on a peer), and leave the GPU usable: the next
normal call on it matches the oracle with a clean status.
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle
from conftest import require_b200
from qtts_b200 import _native as nat
from qtts_b200.quant import kernels as qk
from qtts_b200.sharded import FusedAllGatherW8Linear

pytestmark = pytest.mark.gpu

WAIT_NS = 1_000_000  # 1 ms


def _case(n, k, m, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    q, s = oracle.quantize_weight_per_channel(w.numpy())
    return x, q, torch.from_numpy(s).to(torch.bfloat16)


@pytest.mark.parametrize("n,k,m,variant", [
    (4096, 2048, 1, None),    # split-K streaming kernel, clusters of 8
    (2048, 6144, 8, None),    # split-K over the longer K
    (2048, 2048, 40, "umma"),  # tcgen05 kernel, split over a cluster
])
def test_allgather_wait_expires_when_a_peer_never_calls(n, k, m, variant):
    require_b200()
    torch.cuda.synchronize()
    nat.device_status(reset=True)
    x, q, s = _case(n, k, m, seed=300 + m)
    xd, qd, sd = x.cuda(), torch.from_numpy(q).cuda(), s.cuda()
    world, ldo = 2, 2 * n
    mine_out = torch.zeros((m, ldo), dtype=torch.bfloat16, device="cuda")
    fake_out = torch.zeros((m, ldo), dtype=torch.bfloat16, device="cuda")
    mine_sig = torch.zeros(2 * world, dtype=torch.int32, device="cuda")
    fake_sig = torch.zeros(2 * world, dtype=torch.int32, device="cuda")
    sync = torch.zeros(2, dtype=torch.int32, device="cuda")
    peer_out = torch.tensor([mine_out.data_ptr(), fake_out.data_ptr()], dtype=torch.int64, device="cuda")
    peer_sig = torch.tensor([mine_sig.data_ptr(), fake_sig.data_ptr()], dtype=torch.int64, device="cuda")
    v = nat.VARIANT_AUTO if variant is None else nat.variant_umma(4)

    old = nat.set_wait_limit_ns(WAIT_NS)
    try:
        t0 = time.perf_counter()
        qk.w8_gemm_allgather(xd, qd, sd, None, peer_out=peer_out, ldo=ldo, col_offset=0, peer_signal=peer_sig,
                             sync=sync, rank=0, world=world, variant=v)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        nat.set_wait_limit_ns(old)
    assert nat.device_status() == nat.ERR_TIMEOUT
    assert elapsed < 5.0, f"the expired call took {elapsed:.2f} s"
    # Nothing stored: the store gate never opened.
    assert not mine_out.any() and not fake_out.any()
    # Both pads hold this rank's "ready" and "done" for call 1 and nothing from the fake rank.
    assert mine_sig.tolist() == [1, 0, 1, 0]
    assert fake_sig.tolist() == [1, 0, 1, 0]
    # The call completed on this rank: count re-armed, epoch 1 recorded.
    assert sync.tolist() == [0, 1]

    # The GPU is usable: a normal call right after matches the oracle.
    nat.device_status(reset=True)
    lin = FusedAllGatherW8Linear(qd, sd, n, max_rows=64)
    out = lin(xd).float().cpu().numpy().astype(np.float64)
    ref = oracle.w8a16_reference(x.float().numpy(), q, s.float().numpy())
    assert oracle.rel_err(out, ref) <= 1e-2
    plain = qk.w8_gemm(xd, qd, sd).float().cpu().numpy()
    assert oracle.rel_err(plain, ref) <= 1e-2
    torch.cuda.synchronize()
    assert nat.device_status() == 0
