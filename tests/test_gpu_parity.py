"""GPU parity of the CUDA matvec path against the reference (via the golden
fixtures and the C restatement), through the C ABI.

Contract (per output element): |y_gpu - y_ref| <= 1e-4 * sum_i |w_i x_i|;
dequantised rows and argmax indices bit-exact.
"""
import os
import subprocess

import numpy as np
import pytest

import oracle as O
from conftest import ROOT, TOL, assert_within_tol
from nedo_gpu import blocks as B

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_dev(lib, torch, t, rows, cols, w, x, batch=1):
    wd, xd = dev(torch, w), dev(torch, np.asarray(x, dtype=np.float32))
    yd = torch.empty((batch, rows) if batch > 1 else rows, dtype=torch.float32, device="cuda")
    lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), batch,
                   torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    lib.status()
    return yd.cpu().numpy()


def test_kat_binary_through_dropin(cuda):
    exe = os.path.join(ROOT, "nedo.cpp_b200", "lib", "test_kernels_gpu")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stdout, r.stderr)


def test_golden_host_api(lib, cuda, golden):
    for name, c in golden.items():
        y = lib.matvec(c["type"], c["rows"], c["cols"], c["w"], c["x"])
        assert_within_tol(y, c["y_native"], c["absdot"], what=name)
    lib.cache_clear()


def test_golden_device_api(lib, cuda, golden):
    for name, c in golden.items():
        y = run_dev(lib, cuda, c["type"], c["rows"], c["cols"], c["w"], c["x"])
        assert_within_tol(y, c["y_native"], c["absdot"], what=name)
        # the reference's own two build flavours differ by far less than the bound
        assert_within_tol(y, c["y_portable"], c["absdot"], what=name + " (portable)")


def test_golden_dequant_bit_exact(lib, cuda, golden):
    for name, c in golden.items():
        wd = dev(cuda, c["w"])
        for k, r in enumerate(c["deq_rows"]):
            out = cuda.empty(c["cols"], dtype=cuda.float32, device="cuda")
            lib.dequant_rows_dev(c["type"], c["rows"], c["cols"], wd.data_ptr(), int(r), 1, out.data_ptr())
            got = out.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), c["deq"][k].view(np.uint32)), (name, r)
            host = lib.embedding_row(c["type"], c["rows"], c["cols"], c["w"], int(r))
            assert np.array_equal(host.view(np.uint32), c["deq"][k].view(np.uint32)), (name, r)
    lib.cache_clear()


SHAPES = [
    (1, 64), (3, 512), (129, 512), (1000, 1536), (257, 2048), (77, 4096), (64, 6144), (40, 14336),
    (9, 30720), (5, 32768), (2, 65536),
]


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0, B.F16])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_seeded_shapes_vs_oracle(lib, cuda, oracle, t, rows, cols):
    seed = rows * 7919 + cols + t
    w = B.gen_weight(t, rows, cols, seed)
    x = B.gen_x(cols, seed)
    y = run_dev(lib, cuda, t, rows, cols, w, x)
    assert_within_tol(y, oracle.matvec(t, rows, cols, w, x), oracle.abs_dot(t, rows, cols, w, x),
                      what=f"{B.TYPE_NAMES[t]} {rows}x{cols}")


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0, B.F16])
def test_generic_path_odd_blocks_and_unaligned(lib, cuda, oracle, t):
    # 3 blocks per row (odd) and an unaligned weight pointer both leave the
    # streaming kernel; the generic kernel must agree too.
    rows, cols = 37, 96
    w = B.gen_weight(t, rows, cols, 5)
    x = B.gen_x(cols, 5)
    y = run_dev(lib, cuda, t, rows, cols, w, x)
    ref, absd = oracle.matvec(t, rows, cols, w, x), oracle.abs_dot(t, rows, cols, w, x)
    assert_within_tol(y, ref, absd, what="odd blocks")
    rows, cols = 50, 512
    w = B.gen_weight(t, rows, cols, 6)
    x = B.gen_x(cols, 6)
    buf = cuda.zeros(w.nbytes + 16, dtype=cuda.uint8, device="cuda")
    buf[2:2 + w.nbytes] = dev(cuda, w.reshape(-1))
    xd = dev(cuda, x)
    yd = cuda.empty(rows, dtype=cuda.float32, device="cuda")
    lib.matvec_dev(t, rows, cols, buf.data_ptr() + 2, xd.data_ptr(), yd.data_ptr(), 1, 0)
    cuda.cuda.synchronize()
    assert_within_tol(yd.cpu().numpy(), oracle.matvec(t, rows, cols, w, x), oracle.abs_dot(t, rows, cols, w, x),
                      what="unaligned")


# The host entry point replays a captured CUDA graph of its call from the second
# call on a weight: repeated calls with new x, interleaved weights, and the same
# weight bytes read as another shape must all match the oracle.
@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0, B.F16])
def test_host_api_repeated_calls(lib, cuda, oracle, t):
    rows, cols = 700, 2048
    wa = B.gen_weight(t, rows, cols, 51)
    wb = B.gen_weight(t, rows, cols, 52)
    for i in range(4):
        for w in (wa, wb):
            x = B.gen_x(cols, 60 + i)
            y = lib.matvec(t, rows, cols, w, x)
            assert_within_tol(y, oracle.matvec(t, rows, cols, w, x), oracle.abs_dot(t, rows, cols, w, x),
                              what=f"call {i}")
    # the same bytes as twice the rows of half the columns
    r2, c2 = 2 * rows, cols // 2
    x = B.gen_x(c2, 70)
    y = lib.matvec(t, r2, c2, wa, x)
    assert_within_tol(y, oracle.matvec(t, r2, c2, wa, x), oracle.abs_dot(t, r2, c2, wa, x), what="reshaped")
    lib.weight_evict(wa)
    lib.weight_evict(wb)


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0, B.F16])
def test_deterministic(lib, cuda, t):
    rows, cols = 3000, 4096
    w = B.gen_weight(t, rows, cols, 11)
    x = B.gen_x(cols, 11)
    a = run_dev(lib, cuda, t, rows, cols, w, x)
    b = run_dev(lib, cuda, t, rows, cols, w, x)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0, B.F16])
def test_batched_matches_serial_reference(lib, cuda, oracle, t):
    rows, cols, batch = 300, 2048, 8
    w = B.gen_weight(t, rows, cols, 21)
    x = B.gen_x(cols, 21, batch=batch)
    y = run_dev(lib, cuda, t, rows, cols, w, x, batch=batch)
    ref = oracle.matvec_batch(t, rows, cols, w, x)
    for b in range(batch):
        assert_within_tol(y[b], ref[b], oracle.abs_dot(t, rows, cols, w, x[b]), what=f"batch item {b}")


# Batches of 16+ vectors with rows shorter than 1024 elements stay on the exact
# int8 kernel (8 tokens per launch).
@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0])
def test_large_batch_short_rows_int8(lib, cuda, oracle, t):
    rows, cols, batch = 19200, 512, 16
    assert lib.plan_info(t, rows, cols, batch)["path"] == 4
    w = B.gen_weight(t, rows, cols, 81)
    x = B.gen_x(cols, 81, batch=batch)
    y = run_dev(lib, cuda, t, rows, cols, w, x, batch=batch)
    ref = oracle.matvec_batch(t, rows, cols, w, x)
    for b in range(batch):
        assert_within_tol(y[b], ref[b], oracle.abs_dot(t, rows, cols, w, x[b]), what=f"token {b}")


# Batches of 2-15 quantised vectors run the int8 tensor-pipe kernel with 8, 4, 2
# and 1 token vectors per launch (every weight unit read once per launch): each
# vector must match the reference's serial matvec.  Shapes cover a ragged last
# tile, rows cut into several column groups (8192 columns) and short rows.
@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0])
@pytest.mark.parametrize("rows,cols,batch", [(333, 2048, 2), (333, 2048, 7), (100, 8192, 13), (4096, 1536, 15),
                                             (1000, 4096, 4)])
def test_small_batch_int8_vs_reference(lib, cuda, oracle, t, rows, cols, batch):
    plan = lib.plan_info(t, rows, cols, batch)
    assert plan["path"] == 4, plan
    w = B.gen_weight(t, rows, cols, 41 + batch)
    x = B.gen_x(cols, 41 + batch, batch=batch)
    y = run_dev(lib, cuda, t, rows, cols, w, x, batch=batch)
    ref = oracle.matvec_batch(t, rows, cols, w, x)
    for b in range(batch):
        assert_within_tol(y[b], ref[b], oracle.abs_dot(t, rows, cols, w, x[b]), what=f"batch item {b}")


# Batches of >= 16 vectors that one multi-vector int8 launch cannot take whole
# run as one tcgen05 GEMM (fp16 x and d*q, fp32 accumulation): the same
# per-element tolerance against the reference's serial matvecs.  Shapes cover ragged token tiles (tiles of 256), ragged row tiles
# (128) and an odd number of 256-element weight chunks.
@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0, B.F16])
# The first three shapes have few 256-row tiles, so their K is split over several
# CTAs (partial sums folded in split order); the last has enough tiles for one
# CTA per tile.
@pytest.mark.parametrize("rows,cols,batch", [(300, 2048, 40), (1000, 4096, 64), (129, 1280, 300), (19200, 2048, 16)])
def test_batched_tensor_core_vs_reference(lib, cuda, oracle, t, rows, cols, batch):
    plan = lib.plan_info(t, rows, cols, batch)
    assert plan["path"] == 5, plan
    w = B.gen_weight(t, rows, cols, 31 + batch)
    x = B.gen_x(cols, 31 + batch, batch=batch)
    y = run_dev(lib, cuda, t, rows, cols, w, x, batch=batch)
    # a second call agrees bit for bit (split-K folds in split order, and its
    # arrival counters are back at zero after every launch)
    again = run_dev(lib, cuda, t, rows, cols, w, x, batch=batch)
    assert np.array_equal(y.view(np.uint32), again.view(np.uint32))
    ref = oracle.matvec_batch(t, rows, cols, w, x)
    for b in range(batch):
        assert_within_tol(y[b], ref[b], oracle.abs_dot(t, rows, cols, w, x[b]), what=f"token {b}")


# Quantised batches of more than 256 tokens run on CTA pairs (256 rows x 512
# tokens per pair, tcgen05 MMAs with M = 256 across the two SMs).  9500 rows
# end inside a pair (the second CTA of the last pair has 32 rows); 520 tokens
# leave a second pair tile with 8 tokens.
@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0])
@pytest.mark.parametrize("rows,cols,batch", [(9500, 1024, 300), (8000, 1024, 520)])
def test_pair_tensor_core_vs_reference(lib, cuda, oracle, t, rows, cols, batch):
    plan = lib.plan_info(t, rows, cols, batch)
    assert plan["path"] == 5, plan
    assert plan["grid"] == 2 * ((rows + 255) // 256) * ((batch + 511) // 512), plan
    w = B.gen_weight(t, rows, cols, 61 + batch)
    x = B.gen_x(cols, 61 + batch, batch=batch)
    y = run_dev(lib, cuda, t, rows, cols, w, x, batch=batch)
    again = run_dev(lib, cuda, t, rows, cols, w, x, batch=batch)
    assert np.array_equal(y.view(np.uint32), again.view(np.uint32))
    ref = oracle.matvec_batch(t, rows, cols, w, x)
    for b in range(batch):
        assert_within_tol(y[b], ref[b], oracle.abs_dot(t, rows, cols, w, x[b]), what=f"token {b}")


# F16 weights go to the tensor-core GEMM from 4 token vectors on (only x is
# rounded to fp16 there); 3 vectors still stream the weight once per vector.
@pytest.mark.parametrize("rows,cols,batch", [(2000, 1536, 5), (300, 2048, 4), (640, 1024, 3)])
def test_f16_small_batch_vs_reference(lib, cuda, oracle, rows, cols, batch):
    t = B.F16
    assert (lib.plan_info(t, rows, cols, batch)["path"] == 5) == (batch >= 4)
    w = B.gen_weight(t, rows, cols, 71 + batch)
    x = B.gen_x(cols, 71 + batch, batch=batch)
    y = run_dev(lib, cuda, t, rows, cols, w, x, batch=batch)
    ref = oracle.matvec_batch(t, rows, cols, w, x)
    for b in range(batch):
        assert_within_tol(y[b], ref[b], oracle.abs_dot(t, rows, cols, w, x[b]), what=f"token {b}")


def test_lm_head_argmax(lib, cuda, oracle):
    # F16 LM head with the greedy pick fused into the matvec kernel.
    rows, cols = 32000, 2048
    w = B.gen_weight(B.F16, rows, cols, 2)
    x = B.gen_x(cols, 2)
    wd, xd = dev(cuda, w), dev(cuda, x)
    yd = cuda.empty(rows, dtype=cuda.float32, device="cuda")
    idx = cuda.full((1,), -1, dtype=cuda.int64, device="cuda")
    val = cuda.zeros(1, dtype=cuda.float32, device="cuda")
    for _ in range(3):  # the scratch counter must reset itself between launches
        lib.matvec_argmax_dev(B.F16, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), idx.data_ptr(),
                              val.data_ptr())
        cuda.cuda.synchronize()
        y = yd.cpu().numpy()
        assert int(idx.item()) == oracle.argmax(y)
        assert val.item() == y[int(idx.item())]
    ref = oracle.matvec(B.F16, rows, cols, w, x)
    assert_within_tol(y, ref, oracle.abs_dot(B.F16, rows, cols, w, x), what="lm head")
    top2 = np.sort(ref)[-2:]
    if top2[1] - top2[0] > 2 * TOL * oracle.abs_dot(B.F16, rows, cols, w, x).max():
        assert int(idx.item()) == oracle.argmax(ref)


def test_argmax_ties_first_index(lib, cuda):
    v = np.zeros(100000, dtype=np.float32)
    v[[777, 5000, 99999]] = 3.0
    vd = dev(cuda, v)
    idx = cuda.full((1,), -1, dtype=cuda.int64, device="cuda")
    lib.argmax_dev(vd.data_ptr(), v.size, idx.data_ptr())
    cuda.cuda.synchronize()
    assert int(idx.item()) == 777


def test_status_clean(lib, cuda):
    lib.status()
