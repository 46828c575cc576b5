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
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from .quant.kernels import w8_gemm

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
