"""The batch-1 int8 kernels of gemv_imma.cu against the C restatement of the
reference (src/kernels.cpp:124-169), per output within 1e-4 * sum|w*x|.

One token vector runs the resident-slice kernel whenever a CTA's share of the
weight fits in shared memory, the ring kernel otherwise; NEDO_GPU_IMMA_SLICE=0
keeps every launch on the ring kernel.  The shapes cover one to ten tiles per
CTA, a partial last tile, fewer tiles than SMs, block-pair counts that are not
a multiple of a work item or of a copy unit, and rows shorter than one unit.
The selection is read once per process, so the ring-kernel run is a child
process."""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, assert_within_tol
from nedo_gpu import blocks as B

pytestmark = pytest.mark.gpu

SHAPES = [(16, 256), (17, 512), (1000, 256), (3000, 768), (300, 1536), (2368, 1536), (2384, 2048), (4096, 4096),
          (11008, 4096), (11840, 4096), (1536, 4096), (4096, 1536), (600, 8192), (5000, 1024), (23000, 1280)]


def _check(lib, orc, torch, t, rows, cols):
    w = B.gen_weight(t, rows, cols, rows + 3 * cols + t)
    x = B.gen_x(cols, rows + t + 1)
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    outs = []
    for _ in range(2):
        yd = torch.full((rows,), float("nan"), device="cuda")
        lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), 1, 0)
        torch.cuda.synchronize()
        lib.status()
        outs.append(yd.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), "not run-to-run identical"
    assert_within_tol(outs[0], orc.matvec(t, rows, cols, w, x), orc.abs_dot(t, rows, cols, w, x),
                      what=f"{B.TYPE_NAMES[t]} {rows}x{cols}")


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_batch1_int8_vs_oracle(lib, oracle, cuda, t, rows, cols):
    _check(lib, oracle, cuda, t, rows, cols)


CHILD = r"""
import sys
sys.path[:0] = [sys.argv[1] + "/oracle", sys.argv[1] + "/nedo.cpp_b200", sys.argv[1] + "/tests"]
import torch
import nedo_gpu, oracle as O
from nedo_gpu import blocks as B
import test_imma_slice_gpu as T
lib = nedo_gpu.load()
orc = O.Oracle()
for t in (B.Q8_0, B.Q4_0):
    for rows, cols in T.SHAPES:
        T._check(lib, orc, torch, t, rows, cols)
print("ok")
"""


def test_ring_kernel_vs_oracle(cuda):
    env = dict(os.environ, NEDO_GPU_IMMA_SLICE="0")
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), (r.stdout[-2000:], r.stderr[-4000:])
