"""nedo_gpu_argmax_dev_noalloc: the argmax entry point that allocates nothing.

It runs the kernel of nedo_gpu_argmax_dev with the per-CTA candidates and the
completion counter in a fixed __device__ array of the library.  These tests
compare it with nedo_gpu_argmax_dev (and numpy's first-index argmax) on the
same device vectors, always with two no-alloc calls in a row: the second call
only works if the first left the counter at zero.  The file name sorts last so
that the suite runs it after every other GPU test; it also passes on its own.
"""
import numpy as np
import pytest

import nedo_gpu

pytestmark = pytest.mark.gpu


def _argmax_pair(lib, torch, vd, n, noalloc):
    idx = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    val = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
    fn = lib.argmax_dev_noalloc if noalloc else lib.argmax_dev
    fn(vd.data_ptr(), n, idx.data_ptr(), val.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return idx, val


def _vector(n, seed, ties=()):
    v = np.random.default_rng(seed).standard_normal(n).astype(np.float32)
    for i in ties:
        if i < n:
            v[i] = np.float32(10.0)
    return v


# n = 1; one CTA; CTA boundaries (1024 elements per CTA); every SM busy; more
# elements than CTAs (strided loop); equal maxima in different CTAs.
CASES = [
    (1, ()),
    (1023, ()),
    (1024, ()),
    (1025, (3, 1024)),
    (148 * 1024, (70000, 5)),
    (148 * 1024 + 1, (148 * 1024, 148 * 1024 - 1)),
    (5_000_003, (4_999_999, 2_500_000, 123_457)),
]


def test_noalloc_first_then_existing(lib, cuda):
    # No other entry point has to run first (in a fresh process this is the
    # library's first call on the device).
    v = _vector(4097, 11)
    vd = cuda.from_numpy(v).cuda()
    a_idx, a_val = _argmax_pair(lib, cuda, vd, v.size, noalloc=True)
    r_idx, r_val = _argmax_pair(lib, cuda, vd, v.size, noalloc=False)
    cuda.cuda.synchronize()
    assert int(a_idx.item()) == int(r_idx.item()) == int(np.argmax(v))
    assert a_val.item() == r_val.item() == v[int(np.argmax(v))]


@pytest.mark.parametrize("n,ties", CASES)
def test_noalloc_matches_existing_entry_point(lib, cuda, n, ties):
    v = _vector(n, 1000 + n, ties)
    vd = cuda.from_numpy(v).cuda()
    r_idx, r_val = _argmax_pair(lib, cuda, vd, n, noalloc=False)
    # two calls in a row on one stream, no synchronisation between them
    a1_idx, a1_val = _argmax_pair(lib, cuda, vd, n, noalloc=True)
    a2_idx, a2_val = _argmax_pair(lib, cuda, vd, n, noalloc=True)
    cuda.cuda.synchronize()
    want = int(np.argmax(v))  # first index of the maximum
    assert int(r_idx.item()) == want
    assert int(a1_idx.item()) == want
    assert int(a2_idx.item()) == want
    assert a1_val.item() == a2_val.item() == r_val.item() == v[want]


def test_noalloc_changing_sizes_back_to_back(lib, cuda):
    # Different CTA counts one after the other on one stream: each launch
    # must find the counter at zero.
    vs = [_vector(n, 7 + n, ties) for n, ties in CASES]
    ds = [cuda.from_numpy(v).cuda() for v in vs]
    outs = [_argmax_pair(lib, cuda, d, v.size, noalloc=True) for v, d in zip(vs, ds)]
    outs += [_argmax_pair(lib, cuda, d, v.size, noalloc=True) for v, d in zip(vs, ds)]
    cuda.cuda.synchronize()
    for k, (idx, _) in enumerate(outs):
        v = vs[k % len(vs)]
        assert int(idx.item()) == int(np.argmax(v))


def test_noalloc_argument_errors(lib, cuda):
    d = cuda.zeros(8, dtype=cuda.float32, device="cuda")
    idx = cuda.zeros(1, dtype=cuda.int64, device="cuda")
    with pytest.raises(nedo_gpu.NedoGpuError, match="argmax of an empty vector") as e:
        lib.argmax_dev_noalloc(d.data_ptr(), 0, idx.data_ptr())
    assert e.value.code == nedo_gpu.ERR_ARG
    with pytest.raises(nedo_gpu.NedoGpuError, match="null pointer"):
        lib.argmax_dev_noalloc(d.data_ptr(), 8, None)
    with pytest.raises(nedo_gpu.NedoGpuError, match="more than 2\\^32-1"):
        lib.argmax_dev_noalloc(d.data_ptr(), 1 << 32, idx.data_ptr())
