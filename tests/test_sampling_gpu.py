"""The LM head's sampling step on the GPU (reference src/model.cpp:33-63).

* nedo_gpu_topk_dev against numpy on random vectors (sizes from one block to a
  vocabulary, k from 1 to 256, equal values, NaN): the k largest by value,
  equal values by smaller index first, NaN never ahead of a number;
* nedo_gpu_lm_head_topk / nedo_gpu_lm_head_argmax (host pointers) against the
  same GPU matvec's logits read back in full;
* the drop-in's nedo::kernels::sample_lm_head against the reference's sampler
  (oracle/sample_ref.hpp) on the same logits and generator seeds
  (tests/sample_parity.cpp): identical tokens and generator states.
"""
import os
import subprocess
import tempfile

import numpy as np
import pytest

import nedo_gpu
from conftest import ROOT
from nedo_gpu import blocks as B

pytestmark = pytest.mark.gpu


def _expected_topk(v, k):
    idx = np.arange(v.size)
    key = np.where(np.isnan(v), -np.inf, v.astype(np.float64))
    nan_last = np.isnan(v).astype(np.int8)
    order = np.lexsort((idx, -key, nan_last))  # NaN last, value desc, index asc
    return order[:k]


@pytest.mark.parametrize("n,k", [(1, 1), (100, 7), (2048, 40), (2049, 256), (128000, 40), (128000, 256),
                                 (300000, 100), (64000, 1)])
def test_topk_matches_numpy(lib, cuda, n, k):
    torch = cuda
    rng = np.random.default_rng(n + k)
    v = rng.standard_normal(n).astype(np.float32)
    if n > 10:
        v[rng.integers(0, n, size=n // 10)] = np.float32(0.5)  # many equal values
        v[rng.integers(0, n, size=3)] = np.nan
    vd = torch.from_numpy(v).cuda()
    ids = torch.empty(k, dtype=torch.int32, device="cuda")
    vals = torch.empty(k, dtype=torch.float32, device="cuda")
    for _ in range(2):  # the merge counter resets itself
        lib.topk_dev(vd.data_ptr(), n, k, ids.data_ptr(), vals.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        got = ids.cpu().numpy().view(np.uint32).astype(np.int64)
        exp = _expected_topk(v, k)
        assert np.array_equal(got, exp), (got[:10], exp[:10])
        assert np.array_equal(vals.cpu().numpy().view(np.uint32), v[exp].view(np.uint32))


def test_topk_argument_errors(lib, cuda):
    torch = cuda
    vd = torch.zeros(10, device="cuda")
    ids = torch.empty(300, dtype=torch.int32, device="cuda")
    for n, k in ((10, 0), (10, 11), (10, 257), (0, 1)):
        with pytest.raises(nedo_gpu.NedoGpuError) as e:
            lib.topk_dev(vd.data_ptr(), n, k, ids.data_ptr())
        assert e.value.code == nedo_gpu.ERR_ARG


@pytest.mark.parametrize("t,rows,cols", [(B.F16, 64000, 1536), (B.Q8_0, 32000, 2048), (B.Q4_0, 5000, 4096)])
def test_lm_head_host_entry_points(lib, cuda, t, rows, cols):
    torch = cuda
    w = B.gen_weight(t, rows, cols, 401)
    x = B.gen_x(cols, 401)
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    yd = torch.empty(rows, device="cuda")
    lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), 1, 0)
    torch.cuda.synchronize()
    logits = yd.cpu().numpy()
    for k in (1, 40, 256):
        ids, vals = lib.lm_head_topk(t, rows, cols, w, x, k)
        exp = _expected_topk(logits, k)
        assert np.array_equal(ids.astype(np.int64), exp)
        assert np.array_equal(vals.view(np.uint32), logits[exp].view(np.uint32))
    # the greedy pick runs the matvec with the argmax fused (for Q8_0 / Q4_0 another
    # kernel than the plain matvec, so its logits may differ in the last bits):
    # bit-exact against the same fused launch on device buffers
    idx, val = lib.lm_head_argmax(t, rows, cols, w, x)
    ya = torch.empty(rows, device="cuda")
    ia = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    lib.matvec_argmax_dev(t, rows, cols, wd.data_ptr(), xd.data_ptr(), ya.data_ptr(), ia.data_ptr())
    torch.cuda.synchronize()
    fused = ya.cpu().numpy()
    assert idx == int(ia.item()) == int(np.argmax(fused)) and val == fused[idx]
    assert idx == int(np.argmax(logits))  # both logit vectors pick the same token here
    lib.weight_evict(w)


def test_sample_lm_head_matches_reference_sampler(cuda):
    exe = os.path.join(tempfile.mkdtemp(prefix="nedo_sample_"), "sample_parity")
    lib_dir = os.path.join(ROOT, "nedo.cpp_b200", "lib")
    subprocess.run(["g++", "-std=c++20", "-O2", "-I", os.path.join(ROOT, "nedo.cpp_b200", "cpp", "compat"),
                    "-I", os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "sample_parity.cpp"),
                    "-L", lib_dir, "-lnedo_kernels_cuda", "-lnedo_gpu", f"-Wl,-rpath,{lib_dir}", "-o", exe],
                   check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.startswith("ok"), (r.returncode, r.stdout, r.stderr)
