"""CPU: pin the C restatement (oracle/nedo_oracle.c) to the reference.

Against the golden fixtures (outputs of the reference's own kernels.cpp, both
build flavours) and, where the reference was compiled here, against the live
library on fresh seeded inputs.  Restatement and reference must agree bit for
bit: the restatement follows the reference's summation order exactly.
"""
import numpy as np
import pytest

import oracle as O
from nedo_gpu import blocks as B


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_golden_matvec_native_bit_exact(oracle, golden):
    for name, c in golden.items():
        y = oracle.matvec(c["type"], c["rows"], c["cols"], c["w"], c["x"], O.NATIVE)
        assert np.array_equal(bits(y), bits(c["y_native"])), name


def test_golden_matvec_portable_bit_exact(oracle, golden):
    for name, c in golden.items():
        y = oracle.matvec(c["type"], c["rows"], c["cols"], c["w"], c["x"], O.PORTABLE)
        assert np.array_equal(bits(y), bits(c["y_portable"])), name


def test_golden_dequant_bit_exact(oracle, golden):
    for name, c in golden.items():
        for k, r in enumerate(c["deq_rows"]):
            row = oracle.embedding_row(c["type"], c["rows"], c["cols"], c["w"], int(r))
            assert np.array_equal(bits(row), bits(c["deq"][k])), (name, r)


def test_reference_kats(oracle, golden):
    # tests/test_kernels.cpp:33-65: y = -16 for both one-block tensors, and the
    # Q4_0 embedding row is i-8 (low nibbles) then 7-i (high nibbles).
    for name in ("kat_q8", "kat_q4"):
        c = golden[name]
        assert c["y_native"][0] == -16.0
        assert oracle.matvec(c["type"], 1, 32, c["w"], c["x"])[0] == -16.0
    row = oracle.embedding_row(B.Q4_0, 1, 32, golden["kat_q4"]["w"], 0)
    assert np.array_equal(row[:16], np.arange(16) - 8.0)
    assert np.array_equal(row[16:], 7.0 - np.arange(16))


def test_fp16_codec(oracle):
    hs = np.arange(65536, dtype=np.uint16)
    ref = hs.view(np.float16).astype(np.float32)
    dec = np.array([oracle.fp16_to_fp32(int(h)) for h in hs[::7]], dtype=np.float32)
    finite = np.isfinite(ref[::7]) | np.isinf(ref[::7])
    assert np.array_equal(bits(dec)[finite], bits(ref[::7])[finite])
    rng = np.random.default_rng(0)
    fs = (rng.standard_normal(5000) * 10.0 ** rng.integers(-8, 5, 5000)).astype(np.float32)
    fs = np.concatenate([fs, np.array([0, 65504, 65519.99, 65520, 6e-8, 2.98e-8], dtype=np.float32)])
    enc = np.array([oracle.fp32_to_fp16(float(f)) for f in fs], dtype=np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(enc, fs.astype(np.float16).view(np.uint16))


def test_blocks_dequant_matches_oracle(oracle):
    for t in (B.F16, B.Q8_0, B.Q4_0):
        rows, cols = 5, 256
        w = B.gen_weight(t, rows, cols, 9)
        full = B.dequant(t, w, rows, cols)
        for r in range(rows):
            assert np.array_equal(bits(full[r]), bits(oracle.embedding_row(t, rows, cols, w, r)))


def test_row_bytes_and_errors():
    assert B.row_bytes(B.Q8_0, 4096) == 4352
    assert B.row_bytes(B.Q4_0, 4096) == 2304
    assert B.row_bytes(B.F16, 2048) == 4096
    with pytest.raises(ValueError, match="not block aligned"):
        B.row_bytes(B.Q4_0, 48)


@pytest.mark.parametrize("t", [B.F16, B.Q8_0, B.Q4_0])
def test_restatement_matches_live_reference(oracle, reference, t):
    for rows, cols, seed in ((300, 1536, 1), (64, 4096, 2), (17, 96, 3)):
        w = B.gen_weight(t, rows, cols, seed)
        x = B.gen_x(cols, seed)
        y = oracle.matvec(t, rows, cols, w, x)
        assert np.array_equal(bits(y), bits(reference.matvec(t, rows, cols, w, x)))
        for r in (0, rows - 1):
            assert np.array_equal(bits(oracle.embedding_row(t, rows, cols, w, r)),
                                  bits(reference.embedding_row(t, rows, cols, w, r)))


def test_reference_error_semantics(reference):
    w = np.zeros(64, dtype=np.uint8)
    with pytest.raises(RuntimeError, match="Q4_0 elements not block aligned"):
        reference.matvec(B.Q4_0, 1, 48, w, np.zeros(48, np.float32))
    with pytest.raises(RuntimeError, match="bad embedding row"):
        reference.embedding_row(B.Q8_0, 1, 32, w, 1)
