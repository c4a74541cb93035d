"""The tcgen05 batch-1 kernel (gemv_tc8.cu, opt-in with NEDO_GPU_TC8=1) against
the C restatement of the reference (src/kernels.cpp:124-169), per output
within 1e-4 * sum|w*x|.  The selection is read once per process, so the
checks run in a child process with the variable set."""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CHILD = r"""
import sys
sys.path[:0] = [sys.argv[1] + "/oracle", sys.argv[1] + "/nedo.cpp_b200", sys.argv[1] + "/tests"]
import numpy as np, torch
import nedo_gpu, oracle as O
from nedo_gpu import blocks as B
from conftest import assert_within_tol
lib = nedo_gpu.load()
orc = O.Oracle()
for t in (B.Q8_0, B.Q4_0):
    for rows, cols in [(16, 256), (17, 512), (300, 1536), (4096, 4096), (11008, 4096), (77, 8192), (1536, 1536)]:
        assert lib.plan_info(t, rows, cols, 1)["path"] == 6
        w = B.gen_weight(t, rows, cols, rows + cols + t)
        x = B.gen_x(cols, rows + t)
        wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
        yd = torch.empty(rows, device="cuda")
        for _ in range(2):
            lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), 1, 0)
            torch.cuda.synchronize()
            lib.status()
            assert_within_tol(yd.cpu().numpy(), orc.matvec(t, rows, cols, w, x), orc.abs_dot(t, rows, cols, w, x),
                              what=f"tc8 {B.TYPE_NAMES[t]} {rows}x{cols}")
    # non-finite activations give NaN, as the reference's sums
    x = B.gen_x(512, 3)
    x[100] = np.nan
    w = B.gen_weight(t, 40, 512, 3)
    y = lib.matvec(t, 40, 512, w, x)
    assert np.all(np.isnan(y))
print("ok")
"""


def test_tc8_kernel_vs_oracle(cuda):
    env = dict(os.environ, NEDO_GPU_TC8="1")
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), (r.stdout[-2000:], r.stderr[-4000:])
