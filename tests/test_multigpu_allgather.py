"""Fused all-gather of a row-sharded matvec on 2 GPUs (skipped with fewer).

Each rank computes its rows with the int8 tensor-pipe kernel, which also
stores them on the other rank over NVLink; after the completion wait every
rank holds the full y.  Checked against the oracle's full matvec with the
per-element tolerance, over several steps (the two gathered buffers
alternate), for Q4_0 and Q8_0.
"""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT, TOL
from nedo_gpu import blocks as B

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, type_, rows, cols, out_dir):
    import sys

    for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "nedo.cpp_b200")):
        sys.path.insert(0, p)
    import datetime

    import torch
    import torch.distributed as dist

    import nedo_gpu
    from nedo_gpu.shard import FusedShardedMatvec

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        lib = nedo_gpu.load()
        w = B.gen_weight(type_, rows, cols, 9)
        fm = FusedShardedMatvec(lib, type_, rows, cols, dev)
        rb = B.row_bytes(type_, cols)
        shard = w.reshape(-1)[rank * fm.rows_local * rb:(rank + 1) * fm.rows_local * rb]
        wd = torch.from_numpy(np.ascontiguousarray(shard)).to(dev)
        outs = []
        for step in range(4):
            x = torch.from_numpy(B.gen_x(cols, 100 + step)).to(dev)
            y = fm.run(wd.data_ptr(), x.data_ptr(), torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            outs.append(y.cpu().numpy().copy())
        lib.status()
        np.save(os.path.join(out_dir, f"y{rank}.npy"), np.stack(outs))
        dist.barrier()
        del fm
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("type_,rows,cols", [(B.Q4_0, 4096, 4096), (B.Q8_0, 2048, 1536)])
def test_fused_allgather_two_gpus(tmp_path, oracle, cuda, type_, rows, cols):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), type_, rows, cols, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    w = B.gen_weight(type_, rows, cols, 9)
    for step in range(4):
        x = B.gen_x(cols, 100 + step)
        ref = oracle.matvec(type_, rows, cols, w, x)
        bound = TOL * oracle.abs_dot(type_, rows, cols, w, x)
        for r in range(world):
            y = np.load(tmp_path / f"y{r}.npy")[step]
            assert np.all(np.abs(y.astype(np.float64) - ref) <= bound), (step, r)
