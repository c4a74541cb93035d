"""GPU checks of the library's failure handling and state (no fault, no trap).

* a bounded wait that runs out: the all-gather completion wait on one GPU,
  with a 10 ms bound and a signal word nothing advances, reports
  NEDO_GPU_ERR_DEVICE through nedo_gpu_status, leaves the device usable, and
  still consumes its step: a late signal of that step does not satisfy the
  next one (it would read stale rows);
* the residency cache of the host entry point: the same host buffer (same
  address and size) with new bytes is uploaded again (content fingerprint);
* a batched call captured in a CUDA graph stays valid after a larger call
  grew the per-device buffers;
* argmax NaN behaviour of std::max_element (src/model.cpp:36): NaNs never
  win, except a NaN at index 0, which is returned; the result is always a
  valid index;
* the host batched entry point (nedo_gpu_matvec_batch) against the
  reference's serial matvecs (src/model.cpp:262-266 runs one per token);
* batched fp16 tensor-core rounding: the worst case (constant positive x,
  same-sign weights) stays within its documented 2^-10 bound, and the exact
  mode meets 1e-4 * sum|w*x| on it.
"""
import numpy as np
import pytest

import nedo_gpu
from conftest import TOL, assert_within_tol
from nedo_gpu import blocks as B

pytestmark = pytest.mark.gpu


def _s(torch):
    return torch.cuda.current_stream().cuda_stream


def test_wait_timeout_reports_and_recovers(lib, cuda, oracle):
    torch = cuda
    words = torch.zeros(2, dtype=torch.int32, device="cuda")  # signal, expected
    sig, exp = words.data_ptr(), words.data_ptr() + 4
    lib.status()  # clean before
    lib.set_wait_limit_ns(10_000_000)  # 10 ms
    try:
        lib.allgather_wait_dev(sig, exp, 5, _s(torch))
        with pytest.raises(nedo_gpu.NedoGpuError) as e:
            lib.status(_s(torch))
        assert e.value.code == nedo_gpu.ERR_DEVICE and "bounded wait" in str(e.value)
        # the timed-out step was consumed: expected advanced by its increment
        assert words.cpu().tolist() == [0, 5]
        # its late signals arrive now; the next step must still wait for its own
        words[0] = 5
        lib.allgather_wait_dev(sig, exp, 5, _s(torch))
        with pytest.raises(nedo_gpu.NedoGpuError):
            lib.status(_s(torch))
        assert words.cpu().tolist() == [5, 10]
        # once that step's signals are in, a wait succeeds without an error
        words[0] = 15
        lib.allgather_wait_dev(sig, exp, 5, _s(torch))
        lib.status(_s(torch))
        assert words.cpu().tolist() == [15, 15]
    finally:
        lib.set_wait_limit_ns(0)
    # the device is usable afterwards
    rows, cols = 777, 4096
    w = B.gen_weight(B.Q4_0, rows, cols, 8)
    x = B.gen_x(cols, 8)
    y = lib.matvec(B.Q4_0, rows, cols, w, x)
    assert_within_tol(y, oracle.matvec(B.Q4_0, rows, cols, w, x), oracle.abs_dot(B.Q4_0, rows, cols, w, x),
                      what="after timeout")
    lib.weight_evict(w)


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0, B.F16])
def test_resident_weight_same_address_new_bytes(lib, cuda, oracle, t):
    rows, cols = 640, 2048
    buf = B.gen_weight(t, rows, cols, 90)
    addr = buf.ctypes.data
    x = B.gen_x(cols, 90)
    y1 = lib.matvec(t, rows, cols, buf, x)
    assert_within_tol(y1, oracle.matvec(t, rows, cols, buf, x), oracle.abs_dot(t, rows, cols, buf, x), what="first")
    # a new model's tensor mapped where the old one was: same address, same size
    buf[...] = B.gen_weight(t, rows, cols, 91)
    assert buf.ctypes.data == addr
    y2 = lib.matvec(t, rows, cols, buf, x)
    assert_within_tol(y2, oracle.matvec(t, rows, cols, buf, x), oracle.abs_dot(t, rows, cols, buf, x),
                      what="rewritten bytes")
    assert not np.array_equal(y1, y2)
    lib.weight_evict(buf)


def test_captured_batch_survives_buffer_growth(lib, cuda, oracle):
    torch = cuda
    t, rows, cols = B.Q8_0, 1000, 4096
    w = B.gen_weight(t, rows, cols, 93)
    wd = torch.from_numpy(w).cuda()
    x40 = B.gen_x(cols, 93, batch=40)
    x64 = B.gen_x(cols, 94, batch=64)
    xd40, xd64 = torch.from_numpy(x40).cuda(), torch.from_numpy(x64).cuda()
    y40 = torch.empty((40, rows), device="cuda")
    y64 = torch.empty((64, rows), device="cuda")
    assert lib.plan_info(t, rows, cols, 40)["path"] == 5
    stream = torch.cuda.Stream()
    lib.reserve(t, rows, cols, 40)  # sized outside capture
    # one eager call first: per-process kernel set-up happens outside capture
    lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd40.data_ptr(), y40.data_ptr(), 40, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd40.data_ptr(), y40.data_ptr(), 40, stream.cuda_stream)
    # a larger call grows the shared buffers (the captured ones are retired, not freed)
    lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd64.data_ptr(), y64.data_ptr(), 64, _s(torch))
    torch.cuda.synchronize()
    y40.zero_()
    graph.replay()
    torch.cuda.synchronize()
    lib.status()
    ref40 = oracle.matvec_batch(t, rows, cols, w, x40)
    got40 = y40.cpu().numpy()
    for b in range(0, 40, 3):
        assert_within_tol(got40[b], ref40[b], oracle.abs_dot(t, rows, cols, w, x40[b]), what=f"replayed token {b}")
    ref64 = oracle.matvec_batch(t, rows, cols, w, x64)
    got64 = y64.cpu().numpy()
    for b in range(0, 64, 7):
        assert_within_tol(got64[b], ref64[b], oracle.abs_dot(t, rows, cols, w, x64[b]), what=f"large token {b}")
    del graph


def _argmax_all(lib, torch, v):
    vd = torch.from_numpy(v).cuda()
    out = []
    for fn in (lib.argmax_dev, lib.argmax_dev_noalloc):
        idx = torch.full((1,), -1, dtype=torch.int64, device="cuda")
        fn(vd.data_ptr(), v.size, idx.data_ptr(), None, _s(torch))
        torch.cuda.synchronize()
        out.append(int(idx.item()))
    return out


def _max_element(v):
    """std::max_element with operator<: keep the first element unless a later one compares greater."""
    best = 0
    for i in range(1, v.size):
        if v[best] < v[i]:
            best = i
    return best


@pytest.mark.parametrize("n", [1, 100, 5000, 300000])
def test_argmax_nan_semantics(lib, cuda, n):
    torch = cuda
    rng = np.random.default_rng(n)
    cases = []
    v = rng.standard_normal(n).astype(np.float32)
    v[0] = np.nan
    cases.append(v)  # NaN first: index 0
    v = rng.standard_normal(n).astype(np.float32)
    v[rng.integers(0, n, size=max(1, n // 10))] = np.nan
    v[0] = -1.0
    cases.append(v)  # NaNs elsewhere never win
    cases.append(np.full(n, np.nan, dtype=np.float32))  # all NaN: index 0
    for v in cases:
        expect = _max_element(v) if n <= 5000 else (0 if np.isnan(v[0]) else int(np.nanargmax(v)))
        assert _argmax_all(lib, torch, v) == [expect, expect]


def test_fused_head_argmax_nan(lib, cuda):
    torch = cuda
    rows, cols = 4096, 2048
    w = B.gen_weight(B.F16, rows, cols, 95).view(np.uint16).copy()
    x = B.gen_x(cols, 95)
    for nan_row in (0, 1234):
        wn = w.copy()
        wn[nan_row, 7] = 0x7E00  # an fp16 NaN: that row's logit is NaN
        wd = torch.from_numpy(wn.view(np.uint8)).cuda()
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty(rows, device="cuda")
        idx = torch.full((1,), -1, dtype=torch.int64, device="cuda")
        lib.matvec_argmax_dev(B.F16, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), idx.data_ptr(),
                              None, _s(torch))
        torch.cuda.synchronize()
        y = yd.cpu().numpy()
        assert np.isnan(y[nan_row])
        expect = 0 if nan_row == 0 else int(np.nanargmax(y))
        assert int(idx.item()) == expect


@pytest.mark.parametrize("t,rows,cols,batch", [(B.Q8_0, 1000, 4096, 512), (B.Q4_0, 700, 2048, 8),
                                               (B.F16, 900, 1536, 16)])
def test_host_batch_entry_point(lib, cuda, oracle, t, rows, cols, batch):
    w = B.gen_weight(t, rows, cols, 96 + batch)
    x = B.gen_x(cols, 96 + batch, batch=batch)
    y = lib.matvec_batch(t, rows, cols, w, x)
    sel = range(0, batch, max(1, batch // 64))
    ref = oracle.matvec_batch(t, rows, cols, w, x[list(sel)])
    for j, b in enumerate(sel):
        assert_within_tol(y[b], ref[j], oracle.abs_dot(t, rows, cols, w, x[b]), what=f"token {b}")
    lib.weight_evict(w)


def _same_sign_q8(rows, cols, seed):
    rng = np.random.default_rng(seed)
    nb = cols // 32
    q = rng.integers(1, 128, size=(rows, nb, 32)).astype(np.int8)
    d = (np.abs(rng.normal(0.0, 0.02, size=(rows, nb))) / 127.0).astype(np.float16)
    return B.pack_q8_0(d, q)


@pytest.mark.parametrize("t", [B.Q8_0, B.F16])
def test_tensor_core_batch_worst_case_rounding(lib, cuda, oracle, t):
    torch = cuda
    rows, cols, batch = 2048, 4096, 32
    w = _same_sign_q8(rows, cols, 97) if t == B.Q8_0 else np.abs(
        B.gen_weight(B.F16, rows, cols, 97).view(np.float16)).view(np.uint8)
    # constant positive activations: fp16(0.1) is 2.4e-4 below 0.1 in every element
    x = np.full((batch, cols), 0.1, dtype=np.float32)
    wd, xd = torch.from_numpy(np.ascontiguousarray(w)).cuda(), torch.from_numpy(x).cuda()
    yd = torch.empty((batch, rows), device="cuda")
    ref = oracle.matvec(t, rows, cols, w, x[0])
    absd = oracle.abs_dot(t, rows, cols, w, x[0])

    def run():
        lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), batch, _s(torch))
        torch.cuda.synchronize()
        lib.status()
        return yd.cpu().numpy()

    assert lib.plan_info(t, rows, cols, batch)["path"] == 5
    fast = run()
    # default fp16 GEMM: inside its documented worst case 2^-10 * sum|w*x|
    assert_within_tol(fast[0], ref, absd, tol=2.0 ** -10, what="fp16 GEMM worst case")
    prev = lib.set_exact_batches(True)
    try:
        assert lib.plan_info(t, rows, cols, batch)["path"] in (3, 4)
        exact = run()
    finally:
        lib.set_exact_batches(prev)
    for b in (0, batch - 1):
        assert_within_tol(exact[b], ref, absd, tol=TOL, what=f"exact mode token {b}")


@pytest.mark.parametrize("t", [B.Q8_0, B.Q4_0, B.F16])
@pytest.mark.parametrize("rows,cols,batch", [(300, 4096, 1), (11008, 4096, 1), (1000, 2048, 8), (1000, 4096, 64)])
def test_nonfinite_activation_gives_nan(lib, cuda, t, rows, cols, batch):
    # the reference's fp32 sums are NaN for every row when x holds a NaN
    torch = cuda
    w = B.gen_weight(t, rows, cols, 98)
    x = B.gen_x(cols, 98, batch=batch)
    x[:, cols // 3] = np.nan
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(np.ascontiguousarray(x)).cuda()
    yd = torch.zeros((batch, rows), device="cuda")
    lib.matvec_dev(t, rows, cols, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), batch, _s(torch))
    torch.cuda.synchronize()
    lib.status()
    assert np.all(np.isnan(yd.cpu().numpy()))
