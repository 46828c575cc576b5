"""Int8 weight-only linear sharded along N across the ranks of a process group.

Output channels of a W8A16 linear are independent: each rank holds rows
``[start, stop)`` of the int8 weight and of its per-channel scale (scales go
with their rows), multiplies the full activation ``x [M, K]`` (replicated on
every rank) by its slice on its own GPU, and the bf16 outputs are all-gathered
over NCCL -- the single exchange step of this path. This is the multi-GPU
form of the standalone GEMM benchmark (config 5: K in {2048, 6144}, N in
{12288, 49152}, M in {1, 8, 64}); the serving engine itself runs independent
data-parallel replicas and does not shard.

Layout: every rank owns ``shard = ceil(N / world)`` rows (the last rank may
own fewer real ones). The gather is rank-major, ``[world, M, shard]``, and
the result is its column-block concatenation ``[M, N]``.

:class:`FusedAllGatherW8Linear` is the same product in one kernel per rank:
the GEMM's epilogue stores its block straight into every rank's gathered
``[M, world * shard]`` buffer over peer memory (CUDA IPC mappings, plain P2P
stores over NVLink) and two flag phases replace the collective
(``qtts_w8a16_gemm_allgather``).
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from .quant.kernels import w8_gemm, w8_gemm_allgather

LocalGemm = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, "torch.Tensor | None"], torch.Tensor]


def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows ``[start, stop)`` of an ``n``-row weight owned by ``rank`` of ``world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    shard = -(-n // world)
    start = min(n, rank * shard)
    return start, min(n, start + shard)


def shard_width(n: int, world: int) -> int:
    return -(-n // world)


class ShardedW8Linear:
    """``x @ (W * scale).T + bias`` with W's rows split over the ranks of ``group``.

    ``weight``/``scale``/``bias`` are this rank's rows (``shard_rows``). The
    local product runs through ``gemm`` (the library's ``w8_gemm`` by default)
    and the outputs are all-gathered. ``__call__`` returns the full ``[M, N]``;
    ``local`` and ``gather`` expose the two steps for timing them separately.
    """

    def __init__(
        self,
        weight: torch.Tensor,
        scale: torch.Tensor,
        n_total: int,
        *,
        bias: torch.Tensor | None = None,
        group: dist.ProcessGroup | None = None,
        gemm: LocalGemm | None = None,
    ) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        start, stop = shard_rows(n_total, self.world, self.rank)
        if weight.shape[0] != stop - start or scale.numel() != stop - start:
            raise ValueError(
                f"rank {self.rank} owns rows [{start}, {stop}) of {n_total}; got weight {tuple(weight.shape)}, "
                f"scale {scale.numel()}"
            )
        self.weight, self.scale, self.bias = weight, scale, bias
        self.n_total = n_total
        self.rows = stop - start
        self.shard = shard_width(n_total, self.world)
        self.gemm = gemm

    def local(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's ``[M, shard]`` block (columns past its real rows are left as they are)."""
        m = x.shape[0]
        if out is None:
            out = torch.zeros((m, self.shard), dtype=x.dtype, device=x.device)
        if self.rows > 0:
            if self.gemm is None:
                # The kernel writes its rows straight into the block (row stride = shard).
                w8_gemm(x, self.weight, self.scale, self.bias, out=out[:, : self.rows])
            else:
                out[:, : self.rows] = self.gemm(x, self.weight, self.scale, self.bias)
        return out

    def gather(self, block: torch.Tensor, gathered: torch.Tensor | None = None) -> torch.Tensor:
        """All-gather the ``[M, shard]`` blocks into ``[world, M, shard]`` (rank-major)."""
        m, shard = block.shape
        if gathered is None:
            gathered = torch.empty((self.world, m, shard), dtype=block.dtype, device=block.device)
        if self.world == 1:
            gathered[0].copy_(block)
        else:
            # The collective takes the concatenated [world * M, shard] form.
            dist.all_gather_into_tensor(gathered.view(self.world * m, shard), block.contiguous(), group=self.group)
        return gathered

    def assemble(self, gathered: torch.Tensor) -> torch.Tensor:
        """``[world, M, shard]`` -> ``[M, N]``: the column blocks side by side."""
        world, m, shard = gathered.shape
        return gathered.permute(1, 0, 2).reshape(m, world * shard)[:, : self.n_total]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.assemble(self.gather(self.local(x)))


Exchange = Callable[[torch.Tensor, "dist.ProcessGroup | None"], "list[torch.Tensor]"]


def exchange_peer_tensors(t: torch.Tensor, group: dist.ProcessGroup | None = None) -> list[torch.Tensor]:
    """Every rank's ``t`` mapped into this process (CUDA IPC), in rank order.

    A collective: each rank shares its tensor's IPC handle through the process
    group and opens the others'. The returned tensors alias the peers' device
    memory; keep them alive as long as the peers' buffers are used.

    Each handle is opened on THIS rank's device (the one whose kernels store
    through it), with peer access enabled on demand -- not on the device index
    the owner recorded, which in a process that sees every GPU would map the
    peer's memory into another device's context, unusable from this one.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return [t]
    from torch.multiprocessing.reductions import rebuild_cuda_tensor, reduce_tensor

    rank = dist.get_rank(group)
    handles: list = [None] * world
    dist.all_gather_object(handles, reduce_tensor(t), group=group)
    out = []
    for q, (rebuild, args) in enumerate(handles):
        if q == rank:
            out.append(t)
            continue
        if rebuild is not rebuild_cuda_tensor:
            raise RuntimeError(f"rank {q} did not share a CUDA tensor")
        # rebuild_cuda_tensor(tensor_cls, size, stride, offset, storage_cls, dtype, storage_device, ...)
        args = list(args)
        args[6] = t.device.index
        out.append(rebuild(*args))
    return out


class FusedAllGatherW8Linear:
    """``x @ (W * scale).T + bias`` with W's rows split over the ranks, gathered in the
    GEMM kernel itself (one launch per rank per call, no separate collective).

    Construction is collective (every rank of ``group``, same ``n_total``,
    ``max_rows`` and dtype): each rank allocates its gathered output
    ``[max_rows, world * shard]``, a signal pad and a call counter, and maps the
    other ranks' buffers through CUDA IPC. ``__call__(x)`` returns this rank's
    gathered output ``[M, n_total]`` (a view of the persistent buffer, valid
    until the next call). Every rank must call with the same ``M`` in the same
    order; calls are CUDA-graph capturable. ``share_from`` reuses another
    instance's gathered buffer, signal pads and call counter (same group,
    ``n_total``, ``max_rows`` and dtype; calls on one stream) instead of
    setting up new ones.
    """

    def __init__(
        self,
        weight: torch.Tensor,
        scale: torch.Tensor,
        n_total: int,
        *,
        max_rows: int,
        bias: torch.Tensor | None = None,
        dtype: torch.dtype = torch.bfloat16,
        group: dist.ProcessGroup | None = None,
        exchange: Exchange | None = None,
        launch: Callable[..., None] | None = None,
        share_from: "FusedAllGatherW8Linear | None" = None,
    ) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        start, stop = shard_rows(n_total, self.world, self.rank)
        if weight.shape[0] != stop - start or scale.numel() != stop - start:
            raise ValueError(
                f"rank {self.rank} owns rows [{start}, {stop}) of {n_total}; got weight {tuple(weight.shape)}, "
                f"scale {scale.numel()}"
            )
        if max_rows < 1:
            raise ValueError("max_rows must be positive")
        if shard_rows(n_total, self.world, self.world - 1)[1] <= shard_rows(n_total, self.world, self.world - 1)[0]:
            raise ValueError(f"{n_total} output channels leave a rank of {self.world} without any")
        self.weight, self.scale, self.bias = weight, scale, bias
        self.n_total = n_total
        self.rows = stop - start
        self.shard = shard_width(n_total, self.world)
        self.ldo = self.world * self.shard
        self.col_offset = self.rank * self.shard
        self.max_rows = max_rows
        device = weight.device
        self._launch = launch or w8_gemm_allgather
        if share_from is not None:
            src = share_from
            if (src.n_total, src.world, src.rank, src.max_rows, src.gathered.dtype) != (
                    n_total, self.world, self.rank, max_rows, dtype):
                raise ValueError("share_from must have the same n_total, world, rank, max_rows and dtype")
            self.gathered, self.signal, self.sync = src.gathered, src.signal, src.sync
            self._peer_gathered, self._peer_signal = src._peer_gathered, src._peer_signal
            self.peer_out, self.peer_sig = src.peer_out, src.peer_sig
            return
        self.gathered = torch.zeros((max_rows, self.ldo), dtype=dtype, device=device)
        self.signal = torch.zeros(2 * self.world, dtype=torch.int32, device=device)
        self.sync = torch.zeros(2, dtype=torch.int32, device=device)
        exchange = exchange or exchange_peer_tensors
        # Keep the peers' mappings alive: the kernel stores through them.
        self._peer_gathered = exchange(self.gathered, group)
        self._peer_signal = exchange(self.signal, group)
        self.peer_out = torch.tensor([t.data_ptr() for t in self._peer_gathered], dtype=torch.int64, device=device)
        self.peer_sig = torch.tensor([t.data_ptr() for t in self._peer_signal], dtype=torch.int64, device=device)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        m = x.shape[0]
        if m > self.max_rows:
            raise ValueError(f"{m} rows exceed max_rows={self.max_rows}")
        if x.dtype != self.gathered.dtype:
            raise ValueError(f"x is {x.dtype}, the gathered buffer {self.gathered.dtype}")
        if m > 0:
            self._launch(
                x, self.weight, self.scale, self.bias,
                peer_out=self.peer_out, ldo=self.ldo, col_offset=self.col_offset,
                peer_signal=self.peer_sig, sync=self.sync, rank=self.rank, world=self.world,
            )
        return self.gathered[:m, : self.n_total]
