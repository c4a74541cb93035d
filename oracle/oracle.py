"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checkers.

* ``Oracle``    -- the C restatement in ``nedo_oracle.c`` (``lib/libnedo_oracle.so``).
* ``Reference`` -- the reference's own ``src/kernels.cpp`` compiled from source by
  ``oracle/Makefile`` into ``_ref/libnedo_ref*.so`` (present only where it was built).

Only tests/, the smoke check and the CPU-baseline leg of bench.py import this
module.  The product (the CUDA library and its host wrappers) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "lib", "libnedo_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libnedo_ref.so")
REF_PORTABLE_LIB = os.path.join(HERE, "_ref", "libnedo_ref_portable.so")

F16, Q4_0, Q8_0 = 1, 2, 8
NATIVE, PORTABLE = 0, 1

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)


def build(force: bool = False) -> None:
    """Run oracle/Makefile (restatement always; the reference when its sources exist)."""
    if force or not os.path.exists(ORACLE_LIB):
        subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def _vp(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def row_bytes(type_: int, cols: int) -> int:
    if type_ == F16:
        return cols * 2
    if type_ == Q4_0:
        return cols // 32 * 18
    if type_ == Q8_0:
        return cols // 32 * 34
    raise ValueError(f"unsupported type {type_}")


class Oracle:
    """The plain-C restatement (always available once ``make -C oracle oracle`` ran)."""

    def __init__(self, path: str = ORACLE_LIB):
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        u32, u64, i32 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        lib.oracle_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        lib.oracle_fp16_to_fp32.restype = ctypes.c_float
        lib.oracle_fp32_to_fp16_rne.argtypes = [ctypes.c_float]
        lib.oracle_fp32_to_fp16_rne.restype = ctypes.c_uint16
        lib.oracle_matvec.argtypes = [i32, u32, u64, u64, ctypes.c_void_p, _f32p, _f32p]
        lib.oracle_matvec_batch.argtypes = [i32, u32, u64, u64, u64, ctypes.c_void_p, _f32p, _f32p]
        lib.oracle_embedding_row.argtypes = [u32, u64, u64, ctypes.c_void_p, u64, _f32p]
        lib.oracle_abs_dot.argtypes = [u32, u64, u64, ctypes.c_void_p, _f32p, _f64p]
        lib.oracle_argmax.argtypes = [_f32p, u64]
        lib.oracle_argmax.restype = ctypes.c_int64
        self.lib = lib

    def fp16_to_fp32(self, h: int) -> float:
        return self.lib.oracle_fp16_to_fp32(h)

    def fp32_to_fp16(self, f: float) -> int:
        return self.lib.oracle_fp32_to_fp16_rne(f)

    def matvec(self, type_, rows, cols, w: np.ndarray, x: np.ndarray, flavour=NATIVE) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(rows, dtype=np.float32)
        rc = self.lib.oracle_matvec(flavour, type_, rows, cols, _vp(w), _fp(x), _fp(y))
        if rc:
            raise RuntimeError(f"oracle_matvec status {rc}")
        return y

    def matvec_batch(self, type_, rows, cols, w, x: np.ndarray, flavour=NATIVE) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        batch = x.shape[0]
        y = np.empty((batch, rows), dtype=np.float32)
        rc = self.lib.oracle_matvec_batch(flavour, type_, rows, cols, batch, _vp(w), _fp(x), _fp(y))
        if rc:
            raise RuntimeError(f"oracle_matvec_batch status {rc}")
        return y

    def embedding_row(self, type_, rows, cols, w, row) -> np.ndarray:
        out = np.empty(cols, dtype=np.float32)
        rc = self.lib.oracle_embedding_row(type_, rows, cols, _vp(w), row, _fp(out))
        if rc:
            raise RuntimeError(f"oracle_embedding_row status {rc}")
        return out

    def abs_dot(self, type_, rows, cols, w, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(rows, dtype=np.float64)
        rc = self.lib.oracle_abs_dot(type_, rows, cols, _vp(w), _fp(x), out.ctypes.data_as(_f64p))
        if rc:
            raise RuntimeError(f"oracle_abs_dot status {rc}")
        return out

    def argmax(self, v: np.ndarray) -> int:
        v = np.ascontiguousarray(v, dtype=np.float32)
        return int(self.lib.oracle_argmax(_fp(v), v.size))


class Reference:
    """The reference's own kernels.cpp, compiled from source (``oracle/_ref``)."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        lib = ctypes.CDLL(path)
        u32, u64 = ctypes.c_uint32, ctypes.c_uint64
        lib.nedo_ref_matvec.argtypes = [u32, u64, u64, ctypes.c_void_p, u64, _f32p, _f32p]
        lib.nedo_ref_embedding_row.argtypes = [u32, u64, u64, ctypes.c_void_p, u64, u32, _f32p]
        lib.nedo_ref_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        lib.nedo_ref_fp16_to_fp32.restype = ctypes.c_float
        lib.nedo_ref_fp32_to_fp16.argtypes = [ctypes.c_float]
        lib.nedo_ref_fp32_to_fp16.restype = ctypes.c_uint16
        lib.nedo_ref_tensor_nbytes.argtypes = [u32, u64, ctypes.POINTER(ctypes.c_uint64)]
        lib.nedo_ref_last_error.restype = ctypes.c_char_p
        lib.nedo_ref_set_num_threads.argtypes = [ctypes.c_int]
        self.lib = lib
        self.path = path

    @staticmethod
    def available(path: str = REF_LIB) -> bool:
        return os.path.exists(path)

    def last_error(self) -> str:
        return self.lib.nedo_ref_last_error().decode()

    def set_threads(self, n: int) -> None:
        self.lib.nedo_ref_set_num_threads(n)

    def threads(self) -> int:
        return self.lib.nedo_ref_num_threads()

    def has_openmp(self) -> bool:
        return bool(self.lib.nedo_ref_has_openmp())

    def tensor_nbytes(self, type_, n) -> int:
        out = ctypes.c_uint64()
        if self.lib.nedo_ref_tensor_nbytes(type_, n, ctypes.byref(out)):
            raise RuntimeError(self.last_error())
        return out.value

    def matvec(self, type_, rows, cols, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(rows, dtype=np.float32)
        if self.lib.nedo_ref_matvec(type_, rows, cols, _vp(w), w.nbytes, _fp(x), _fp(y)):
            raise RuntimeError(self.last_error())
        return y

    def embedding_row(self, type_, rows, cols, w, row) -> np.ndarray:
        out = np.empty(cols, dtype=np.float32)
        if self.lib.nedo_ref_embedding_row(type_, rows, cols, _vp(w), w.nbytes, row, _fp(out)):
            raise RuntimeError(self.last_error())
        return out

    def fp16_to_fp32(self, h: int) -> float:
        return self.lib.nedo_ref_fp16_to_fp32(h)

    def fp32_to_fp16(self, f: float) -> int:
        return self.lib.nedo_ref_fp32_to_fp16(f)
