"""The multi-GPU host logic (row sharding + all-gather of y) on CPU: two gloo
ranks, each computing its row range with the oracle, must reproduce the
full matvec exactly (rows are independent, so the gathered y is bit-equal).
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT  # noqa: F401  (puts the package and oracle on sys.path)
from nedo_gpu import blocks as B
from nedo_gpu.shard import row_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, type_, rows, cols, out_dir):
    import sys

    for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "nedo.cpp_b200")):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    import oracle as O
    from nedo_gpu.shard import ShardedMatvec

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        orc = O.Oracle()
        w = B.gen_weight(type_, rows, cols, 5)
        x = B.gen_x(cols, 5)
        sm = ShardedMatvec(type_, rows, cols)
        w_shard = sm.shard_bytes(w.reshape(-1))

        def local(xv, y_local):
            y_local.copy_(torch.from_numpy(orc.matvec(type_, sm.rows_local, cols, w_shard, xv)))

        y_local = torch.empty(sm.rows_local, dtype=torch.float32)
        y_full = torch.empty(rows, dtype=torch.float32)
        sm.run(local, x, y_local, y_full)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y_full.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("type_,rows,cols", [(B.Q8_0, 96, 256), (B.Q4_0, 64, 512), (B.F16, 40, 128)])
def test_two_rank_shard_gather_equals_full(tmp_path, oracle, type_, rows, cols):
    world = 2
    port = _free_port()
    mp.start_processes(_rank_main, args=(world, port, type_, rows, cols, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    full = oracle.matvec(type_, rows, cols, B.gen_weight(type_, rows, cols, 5), B.gen_x(cols, 5))
    for r in range(world):
        y = np.load(tmp_path / f"y{r}.npy")
        assert np.array_equal(y, full), f"rank {r}"


def test_row_range_partition():
    for rows in (1, 7, 11008, 32768):
        for world in (1, 2, 3, 8):
            spans = [row_range(rows, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
    with pytest.raises(ValueError):
        row_range(10, 2, 2)
