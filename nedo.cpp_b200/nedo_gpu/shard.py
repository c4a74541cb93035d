"""Row-sharded matvec over several GPUs (one process per GPU).

Rows of a matvec are independent (reference src/kernels.cpp:166-168: each
y[r] depends on row r only), so a matrix splits into contiguous row ranges
with no exchange during the product.  The only collective is the all-gather
of the fp32 y slices (NCCL over NVLink on GPUs; any torch.distributed backend
works, which is how the CPU tests run it with gloo).

    sm = ShardedMatvec(type_, rows_total, cols, group=None)
    begin, end = sm.rows_of(rank)       # this rank's rows
    sm.run(local, x, y_local, y_full)   # local(x, y_local) fills the slice, then all-gather

`local` is the per-rank product: on a GPU the library call
(`Library.matvec_dev` on this rank's weight shard), in tests a CPU function.
"""
from __future__ import annotations

from dataclasses import dataclass

from .blocks import row_bytes


def row_range(rows_total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous even split: rank r owns rows [r*rows/world, (r+1)*rows/world)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    return rows_total * rank // world, rows_total * (rank + 1) // world


@dataclass
class ShardedMatvec:
    type_: int
    rows_total: int
    cols: int
    group: object = None  # torch.distributed process group (None = default)

    def __post_init__(self):
        import torch.distributed as dist

        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.rows_total % self.world:
            # all_gather_into_tensor needs equal slices
            raise ValueError(f"{self.rows_total} rows do not split evenly over {self.world} ranks")
        self.rows_local = self.rows_total // self.world
        self.row_bytes = row_bytes(self.type_, self.cols)

    def rows_of(self, rank: int) -> tuple[int, int]:
        return row_range(self.rows_total, self.world, rank)

    def shard_bytes(self, w_full_bytes):
        """This rank's slice of a full weight (bytes of its row range)."""
        b, e = self.rows_of(self.rank)
        return w_full_bytes[b * self.row_bytes:e * self.row_bytes]

    def run(self, local, x, y_local, y_full):
        """local(x, y_local) computes this rank's rows; then every rank gets all of y."""
        import torch.distributed as dist

        if y_local.numel() != self.rows_local or y_full.numel() != self.rows_total:
            raise ValueError("y buffers do not match the shard sizes")
        local(x, y_local)
        dist.all_gather_into_tensor(y_full, y_local, group=self.group)
        return y_full
