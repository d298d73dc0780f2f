"""Token-sharded tensor-ring operator: one process per GPU, cores replicated.

The benchmark's large-prefill configuration (4096 -> 14336, modes (16,16,16) -> (16,28,32),
rank 16, bf16, 65,536 tokens over 1/2/4/8 GPUs) splits x by rows.  Tokens are independent --
row t of y depends only on row t of x and the cores -- so rank g of G runs the single-GPU
operator on rows [start_g, stop_g) with its own replica of the packed cores, and nothing
crosses NVLink on the data path.  ``gather=True`` adds one all_gather of y for callers that
want every row on every rank; it is a separate, optional step (the bench times it apart from
the kernel).

    op = ShardedRing(cores, spec)          # after torch.distributed.init_process_group
    y_rows = op(x)                         # x: all T rows (same on every rank) -> this rank's rows
    y_all = op(x, gather=True)             # every rank gets all T rows

The split gives the first T % G ranks one extra row; a rank can hold zero rows (T < G).
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .spec import TRSpec


def shard_bounds(tokens: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [start, stop) of `tokens` that rank `rank` of `world` owns (balanced, in order)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if tokens < 0:
        raise ValueError(f"negative token count {tokens}")
    base, extra = divmod(tokens, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class ShardedRing:
    """This rank's share of a token-sharded tensor-ring operator.

    `op_factory(cores, spec)` builds the per-rank operator; the default is this package's
    `prepare_optimized`, which runs the CUDA kernels on the cores' device.  The process group
    (default: the world group) is used only by `gather=True`.
    """

    def __init__(self, cores: Sequence[torch.Tensor], spec: TRSpec,
                 group: Optional[dist.ProcessGroup] = None,
                 op_factory: Optional[Callable] = None):
        if op_factory is None:
            from .ring import prepare_optimized as op_factory
        self.spec = spec
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.fn = op_factory(cores, spec)

    def bounds(self, tokens: int) -> Tuple[int, int]:
        return shard_bounds(tokens, self.world, self.rank)

    def local(self, x_rows: torch.Tensor) -> torch.Tensor:
        """The operator on rows this rank already holds (no slicing, no communication)."""
        return self.fn(x_rows)

    def __call__(self, x: torch.Tensor, gather: bool = False) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != self.spec.in_features:
            raise ValueError(f"x must be [T, {self.spec.in_features}], got {tuple(x.shape)}")
        T = x.shape[0]
        start, stop = self.bounds(T)
        y_rows = self.fn(x[start:stop])
        if not gather or self.world == 1:
            return y_rows
        # all_gather needs equal sizes: pad every share to the largest, then drop the padding
        rows_max = shard_bounds(T, self.world, 0)[1]
        padded = y_rows.new_zeros((rows_max, self.spec.out_features))
        padded[: stop - start] = y_rows
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        dist.all_gather(parts, padded, group=self.group)
        return torch.cat([p[: b - a] for p, (a, b) in
                          zip(parts, (shard_bounds(T, self.world, g) for g in range(self.world)))])
