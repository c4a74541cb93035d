"""Small batches on the multi-vector resident slice of gemv_imma.cu against the
C restatement of the reference (src/kernels.cpp:124-169): every output of every
token vector within 1e-4 * sum|w*x|, and two runs bit-identical.

A batch of 2 to 15 vectors, a batch of up to 32 that one launch takes whole,
and in exact mode any batch, runs as launches of up to 32 vectors; each launch
is split into token groups of 2, 4 or 8 vectors, one group of CTAs per group
of vectors.  The shapes cover one to eight tiles
per CTA, fewer tiles than CTAs, a last copy unit and a last work item that are
partial, and rows the kernel does not take (the ring kernel then runs).  The
batches cover a group-size remainder (odd batches end on the one-vector
kernel) and launches of 16.  NEDO_GPU_IMMA_MULTI fixes the group size; it is
read once per process, so the runs with 4 and 8 vectors per group are child
processes."""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, assert_within_tol
from nedo_gpu import blocks as B

pytestmark = pytest.mark.gpu

SHAPES = [(1536, 1536), (4096, 1536), (1536, 4096), (4096, 4096), (300, 1536), (1000, 1280), (333, 1088),
          (2384, 2048), (17, 512), (11008, 4096)]
BATCHES = [2, 3, 5, 8, 11]


def _check(lib, orc, torch, t, rows, cols, batch):
    w = B.gen_weight(t, rows, cols, rows + 5 * cols + t)
    x = B.gen_x(cols, rows + t + 7, batch=batch)
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(np.ascontiguousarray(x)).cuda()
    outs = []
    for _ in range(2):
        yd = torch.full((batch, rows), float("nan"), device="cuda")
        lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), batch, 0)
        torch.cuda.synchronize()
        lib.status()
        outs.append(yd.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), "not run-to-run identical"
    for k in range(batch):
        assert_within_tol(outs[0][k], orc.matvec(t, rows, cols, w, x[k]), orc.abs_dot(t, rows, cols, w, x[k]),
                          what=f"{B.TYPE_NAMES[t]} {rows}x{cols} batch {batch} vector {k}")


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_small_batches_vs_oracle(lib, oracle, cuda, t, rows, cols):
    for batch in BATCHES:
        _check(lib, oracle, cuda, t, rows, cols, batch)


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0])
def test_exact_mode_batches_of_16_and_more(lib, oracle, cuda, t):
    # exact mode keeps batches of 16 and more off the fp16 GEMM: launches of 16 vectors
    prev = lib.set_exact_batches(True)
    try:
        for rows, cols in [(1536, 1536), (4096, 1536)]:
            _check(lib, oracle, cuda, t, rows, cols, 16)
            _check(lib, oracle, cuda, t, rows, cols, 19)
    finally:
        lib.set_exact_batches(prev)


@pytest.mark.parametrize("t,rows,cols,batch", [(B.Q8_0, 1536, 1536, 16), (B.Q8_0, 1536, 1536, 32),
                                                (B.Q4_0, 1536, 1536, 32), (B.Q8_0, 4096, 1536, 16),
                                                (B.Q4_0, 4096, 1536, 16), (B.Q4_0, 1536, 4096, 16)])
def test_whole_batch_in_one_launch(lib, oracle, cuda, t, rows, cols, batch):
    # batches of 16 to 32 that one multi-vector launch takes stay off the fp16 GEMM
    info = lib.plan_info(t, rows, cols, batch)
    assert info["path"] == 4 and info["launches"] == 1, info
    _check(lib, oracle, cuda, t, rows, cols, batch)


def test_plan_reports_the_multi_vector_launch(lib, cuda):
    # 1536x1536 Q8_0 at 8 vectors: 2 groups of 4 vectors over 74 CTAs each
    info = lib.plan_info(B.Q8_0, 1536, 1536, 8)
    assert info["path"] == 4 and info["grid"] == 148 and info["warps"] == 16 and info["launches"] == 1, info
    # 11 vectors: launches of 10 and 1
    assert lib.plan_info(B.Q8_0, 1536, 1536, 11)["launches"] == 2


CHILD = r"""
import sys
sys.path[:0] = [sys.argv[1] + "/oracle", sys.argv[1] + "/nedo.cpp_b200", sys.argv[1] + "/tests"]
import torch
import nedo_gpu, oracle as O
from nedo_gpu import blocks as B
import test_imma_multi_gpu as T
lib = nedo_gpu.load()
orc = O.Oracle()
for t in (B.Q8_0, B.Q4_0):
    for rows, cols in T.SHAPES:
        for batch in (4, 8, 12):
            T._check(lib, orc, torch, t, rows, cols, batch)
print("ok")
"""


@pytest.mark.parametrize("per_group", ["4", "8", "0"])
def test_group_sizes_vs_oracle(cuda, per_group):
    # "0": the ring kernel for every batch
    env = dict(os.environ, NEDO_GPU_IMMA_MULTI=per_group)
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), (r.stdout[-2000:], r.stderr[-4000:])
