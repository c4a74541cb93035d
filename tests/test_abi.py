"""CPU: the C-ABI library loads, exports every declared symbol, and rejects bad
arguments with the reference's messages before touching a GPU."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import nedo_gpu
from nedo_gpu import blocks as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nedo_gpu.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"NEDO_GPU_API\s+[\w\s\*]+?\b(nedo_gpu_\w+)\s*\(", text)))


def test_header_declares_binding_exports():
    assert declared_symbols() == sorted(nedo_gpu.EXPORTS)


def test_library_exports_every_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", lib.path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (nedo_gpu_\w+)", out))
    for name in declared_symbols():
        assert name in exported, name
        assert hasattr(lib.lib, name)


def test_library_has_no_torch_or_oracle_dependency(lib):
    out = subprocess.run(["ldd", lib.path], capture_output=True, text=True).stdout
    assert "torch" not in out and "oracle" not in out and "nedo_ref" not in out


def test_version(lib):
    assert lib.version() >= 100


@pytest.mark.parametrize("type_,cols,code,msg", [
    (B.Q4_0, 48, nedo_gpu.ERR_ALIGN, "Q4_0 elements not block aligned"),
    (B.Q8_0, 40, nedo_gpu.ERR_ALIGN, "Q8_0 elements not block aligned"),
    (0, 64, nedo_gpu.ERR_TYPE, "matvec tensor type not supported"),
    (30, 64, nedo_gpu.ERR_TYPE, "matvec tensor type not supported"),
    (12, 256, nedo_gpu.ERR_TYPE, "tensor type not implemented: 12"),
])
def test_matvec_argument_errors(lib, type_, cols, code, msg):
    w = np.zeros(4096, dtype=np.uint8)
    x = np.zeros(cols, dtype=np.float32)
    with pytest.raises(nedo_gpu.NedoGpuError, match=re.escape(msg)) as e:
        lib.matvec(type_, 2, cols, w, x)
    assert e.value.code == code


def test_embedding_row_errors(lib):
    w = np.zeros(4096, dtype=np.uint8)
    with pytest.raises(nedo_gpu.NedoGpuError, match="bad embedding row") as e:
        lib.embedding_row(B.Q8_0, 2, 32, w, 2)
    assert e.value.code == nedo_gpu.ERR_ROW
    with pytest.raises(nedo_gpu.NedoGpuError, match="embedding type unsupported"):
        lib.embedding_row(0, 2, 32, w, 0)


def test_short_span_rejected(lib):
    w = np.zeros(33, dtype=np.uint8)  # one Q8_0 block needs 34 bytes
    with pytest.raises(nedo_gpu.NedoGpuError, match="shorter") as e:
        lib.matvec(B.Q8_0, 1, 32, w, np.zeros(32, np.float32))
    assert e.value.code == nedo_gpu.ERR_ARG


def test_zero_rows_is_a_noop(lib):
    # rows == 0: the reference's loop body never runs, so even F32 is accepted.
    y = lib.matvec(B.Q8_0, 0, 64, np.zeros(0, np.uint8), np.zeros(64, np.float32))
    assert y.size == 0
    lib.matvec(0, 0, 64, np.zeros(0, np.uint8), np.zeros(64, np.float32))


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(FileNotFoundError, match="no CPU fallback"):
        nedo_gpu.Library(str(tmp_path / "libnedo_gpu.so"))


def test_dropin_layer_and_kat_binary_built():
    libdir = os.path.join(ROOT, "nedo.cpp_b200", "lib")
    assert os.path.exists(os.path.join(libdir, "libnedo_kernels_cuda.so"))
    assert os.access(os.path.join(libdir, "test_kernels_gpu"), os.X_OK)
    # the drop-in layer exports the reference's C++ entry points
    out = subprocess.run(["nm", "-DC", "--defined-only", os.path.join(libdir, "libnedo_kernels_cuda.so")],
                         capture_output=True, text=True, check=True).stdout
    assert "nedo::kernels::matvec(nedo::TensorInfo const&, std::span<std::byte const, 18446744073709551615ul>, float const*, float*)" in out
    assert "nedo::kernels::embedding_row(" in out
