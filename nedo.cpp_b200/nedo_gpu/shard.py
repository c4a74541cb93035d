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


class FusedShardedMatvec:
    """Row-sharded matvec with the all-gather fused into the kernel (GPUs only).

    The gathered y (and the counter words) live in torch symmetric memory, so
    every rank holds device pointers to every peer's copy.  Each step the int8 tensor-pipe matvec
    stores its rows into all copies over NVLink and counts its CTAs on each
    peer's signal word; a one-thread wait kernel then holds this rank's stream
    until all peers' rows have arrived.  Two gathered buffers alternate by
    step, so a fast rank never overwrites rows a slower rank is still reading
    (the next use of a buffer waits for every rank's previous step).

        fm = FusedShardedMatvec(lib, type_, rows_total, cols, device)
        y_full = fm.run(w_ptr, x_ptr, stream)   # a view of this step's buffer
    """

    def __init__(self, lib, type_, rows_total, cols, device, group=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.lib, self.type_, self.rows_total, self.cols = lib, type_, rows_total, cols
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if rows_total % self.world:
            raise ValueError(f"{rows_total} rows do not split evenly over {self.world} ranks")
        self.rows_local = rows_total // self.world
        plan = lib.plan_info(type_, self.rows_local, cols)
        if plan["path"] != 4:
            raise ValueError("the fused all-gather needs a Q8_0/Q4_0 shape of the int8 tensor-pipe kernel")
        # [gathered y, buffer 0][gathered y, buffer 1][16 words: signal 0, 1; expected 8, 9],
        # zeroed before the rendezvous (a collective: no peer counts on it earlier)
        self.buf = symm.empty(2 * rows_total + 16, dtype=torch.float32, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.handle = symm.rendezvous(self.buf, self.group)
        peers = [k for k in range(self.world) if k != self.rank]
        bp = self.handle.buffer_ptrs
        words = 4 * 2 * rows_total  # byte offset of the counter words
        self.peer_y = [[bp[k] + 4 * b * rows_total for k in peers] for b in (0, 1)]
        self.peer_signal = [[bp[k] + words + 4 * b for k in peers] for b in (0, 1)]
        self.signal = [bp[self.rank] + words + 4 * b for b in (0, 1)]
        self.expected = [bp[self.rank] + words + 4 * (8 + b) for b in (0, 1)]
        self.increment = len(peers) * plan["grid"]
        self.step = 0

    def run(self, w_ptr, x_ptr, stream=0):
        b = self.step & 1
        self.step += 1
        y_full = self.buf[b * self.rows_total:(b + 1) * self.rows_total]
        y_local = y_full.data_ptr() + 4 * self.rank * self.rows_local
        self.lib.matvec_allgather_dev(self.type_, self.rows_local, self.cols, w_ptr, x_ptr, y_local,
                                      self.peer_y[b], self.peer_signal[b], self.rank * self.rows_local, stream)
        self.lib.allgather_wait_dev(self.signal[b], self.expected[b], self.increment, stream)
        return y_full
