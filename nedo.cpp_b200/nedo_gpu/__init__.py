"""Python host binding of libnedo_gpu.so (the C ABI in include/nedo_gpu.h).

The reference exposes this path as C++ (``nedo::kernels::matvec`` /
``embedding_row``, include/nedo/kernels.hpp:20-21); the functions here mirror
those two calls -- same argument meaning (GGUF type code, ``cols`` = shape[0]
contiguous, ``rows`` = shape[1]) and the same error messages -- for tests,
benchmarks and Python callers.  There is no CPU fallback: importing this module
without the built library raises.

Host-pointer calls (``matvec``, ``embedding_row``) take numpy arrays and are
synchronous.  Device calls (``matvec_dev`` ...) take raw device addresses (for
example ``torch.Tensor.data_ptr()``) and a CUDA stream handle, and are
asynchronous on that stream.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import blocks
from .blocks import F16, Q4_0, Q8_0, row_bytes

__all__ = ["F16", "Q4_0", "Q8_0", "row_bytes", "blocks", "Library", "load", "NedoGpuError", "LIB_PATH"]

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(os.path.dirname(HERE), "lib")
LIB_PATH = os.path.join(LIB_DIR, "libnedo_gpu.so")

OK, ERR_TYPE, ERR_ALIGN, ERR_ROW, ERR_ARG, ERR_CUDA, ERR_DEVICE, ERR_NOMEM = range(8)

# Every symbol include/nedo_gpu.h declares (checked by the CPU test suite).
EXPORTS = (
    "nedo_gpu_version",
    "nedo_gpu_set_pdl",
    "nedo_gpu_set_exact_batches",
    "nedo_gpu_last_error",
    "nedo_gpu_set_wait_limit_ns",
    "nedo_gpu_matvec",
    "nedo_gpu_matvec_batch",
    "nedo_gpu_embedding_row",
    "nedo_gpu_weight_upload",
    "nedo_gpu_weight_evict",
    "nedo_gpu_cache_clear",
    "nedo_gpu_matvec_dev",
    "nedo_gpu_reserve",
    "nedo_gpu_matvec_argmax_dev",
    "nedo_gpu_argmax_dev",
    "nedo_gpu_argmax_dev_noalloc",
    "nedo_gpu_topk_dev",
    "nedo_gpu_lm_head_topk",
    "nedo_gpu_lm_head_argmax",
    "nedo_gpu_matvec_allgather_dev",
    "nedo_gpu_allgather_wait_dev",
    "nedo_gpu_dequant_rows_dev",
    "nedo_gpu_status",
    "nedo_gpu_plan_info",
    "nedo_gpu_decoder_create",
    "nedo_gpu_decoder_forward",
    "nedo_gpu_decoder_generate",
    "nedo_gpu_decoder_set_stream",
    "nedo_gpu_decoder_logits_dev",
    "nedo_gpu_decoder_reset",
    "nedo_gpu_decoder_destroy",
)


class NedoGpuError(RuntimeError):
    """A non-zero status from the C ABI; ``code`` is the NEDO_GPU_ERR_* value."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_u32, _u64, _i32, _vp = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_void_p
_f32p = ctypes.POINTER(ctypes.c_float)
_u64p = ctypes.POINTER(ctypes.c_uint64)

class DecoderConfig(ctypes.Structure):
    """nedo_gpu_decoder_config (ModelConfig, include/nedo/model.hpp:12-16)."""
    _fields_ = [(n, ctypes.c_uint32) for n in ("vocab", "dim", "layers", "heads", "kv_heads", "head_dim", "ffn",
                                                "context", "sliding", "morph_layers", "morph_shared", "morph_root",
                                                "morph_suffix")] + [("rms_eps", ctypes.c_float),
                                                                    ("rope_theta", ctypes.c_float)]


class TensorView(ctypes.Structure):
    """nedo_gpu_tensor_view: a GGUF tensor's type, shape and host bytes."""
    _fields_ = [("type", ctypes.c_uint32), ("ndims", ctypes.c_uint32), ("shape", ctypes.c_uint64 * 2),
                ("data", ctypes.c_void_p), ("nbytes", ctypes.c_uint64)]


_SIGNATURES = {
    "nedo_gpu_version": ([], _i32),
    "nedo_gpu_set_pdl": ([_i32], _i32),
    "nedo_gpu_set_exact_batches": ([_i32], _i32),
    "nedo_gpu_last_error": ([], ctypes.c_char_p),
    "nedo_gpu_set_wait_limit_ns": ([_u64], _i32),
    "nedo_gpu_matvec": ([_u32, _u64, _u64, _vp, _u64, _vp, _vp], _i32),
    "nedo_gpu_matvec_batch": ([_u32, _u64, _u64, _vp, _u64, _vp, _vp, _u32], _i32),
    "nedo_gpu_embedding_row": ([_u32, _u64, _u64, _vp, _u64, _u32, _vp], _i32),
    "nedo_gpu_weight_upload": ([_vp, _u64, ctypes.POINTER(_vp)], _i32),
    "nedo_gpu_weight_evict": ([_vp], _i32),
    "nedo_gpu_cache_clear": ([], _i32),
    "nedo_gpu_matvec_dev": ([_u32, _u64, _u64, _vp, _vp, _vp, _u32, _vp], _i32),
    "nedo_gpu_reserve": ([_u32, _u64, _u64, _u32], _i32),
    "nedo_gpu_matvec_argmax_dev": ([_u32, _u64, _u64, _vp, _vp, _vp, _vp, _vp, _vp], _i32),
    "nedo_gpu_argmax_dev": ([_vp, _u64, _vp, _vp, _vp], _i32),
    "nedo_gpu_argmax_dev_noalloc": ([_vp, _u64, _vp, _vp, _vp], _i32),
    "nedo_gpu_topk_dev": ([_vp, _u64, _u32, _vp, _vp, _vp], _i32),
    "nedo_gpu_lm_head_topk": ([_u32, _u64, _u64, _vp, _u64, _vp, _u32, _vp, _vp], _i32),
    "nedo_gpu_lm_head_argmax": ([_u32, _u64, _u64, _vp, _u64, _vp, _vp, _vp], _i32),
    "nedo_gpu_matvec_allgather_dev": ([_u32, _u64, _u64, _vp, _vp, _vp, _u64p, _u64p, _u32, _u64, _vp], _i32),
    "nedo_gpu_allgather_wait_dev": ([_vp, _vp, _u32, _vp], _i32),
    "nedo_gpu_dequant_rows_dev": ([_u32, _u64, _u64, _vp, _u64, _u64, _vp, _vp], _i32),
    "nedo_gpu_status": ([_vp], _i32),
    "nedo_gpu_plan_info": ([_u32, _u64, _u64, _u32, ctypes.POINTER(_u32), _i32], _i32),
    "nedo_gpu_decoder_create": ([ctypes.POINTER(DecoderConfig), ctypes.POINTER(TensorView), _u64, ctypes.POINTER(_vp)],
                                _i32),
    "nedo_gpu_decoder_forward": ([_vp, _u32, _u64, _vp, ctypes.POINTER(_u32)], _i32),
    "nedo_gpu_decoder_generate": ([_vp, _u32, _u64, _u32, _vp], _i32),
    "nedo_gpu_decoder_set_stream": ([_vp, _vp], _i32),
    "nedo_gpu_decoder_logits_dev": ([_vp, ctypes.POINTER(_vp)], _i32),
    "nedo_gpu_decoder_reset": ([_vp], _i32),
    "nedo_gpu_decoder_destroy": ([_vp], None),
}


class Library:
    """ctypes view of libnedo_gpu.so with checked calls."""

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(
                f"{path} is missing: build it with `make -C nedo.cpp_b200` (there is no CPU fallback)")
        self.path = path
        self.lib = ctypes.CDLL(path)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.argtypes = args
            fn.restype = res

    # ------------------------------------------------------------------ utils
    def version(self) -> int:
        return self.lib.nedo_gpu_version()

    def set_pdl(self, enable: bool) -> bool:
        """Programmatic dependent launch for the device entry points; returns the old setting."""
        return bool(self.lib.nedo_gpu_set_pdl(1 if enable else 0))

    def set_exact_batches(self, enable: bool) -> bool:
        """Batched calls on the exact kernels only (no fp16 tensor-core GEMM); returns the old setting."""
        return bool(self.lib.nedo_gpu_set_exact_batches(1 if enable else 0))

    def last_error(self) -> str:
        return self.lib.nedo_gpu_last_error().decode()

    def set_wait_limit_ns(self, ns: int) -> None:
        """Bound of the kernels' spin-waits on the current device (0 = default 2 s)."""
        self._check(self.lib.nedo_gpu_set_wait_limit_ns(ns))

    def _check(self, rc: int) -> None:
        if rc != OK:
            raise NedoGpuError(rc, self.last_error())

    # ------------------------------------------------------- host entry points
    def matvec(self, type_: int, rows: int, cols: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        """nedo::kernels::matvec: y[r] = dot(row r, x).  w holds the GGUF bytes."""
        if not (isinstance(w, np.ndarray) and w.flags.c_contiguous):
            w = np.ascontiguousarray(w)
        if not (isinstance(x, np.ndarray) and x.dtype == np.float32 and x.flags.c_contiguous):
            x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(rows, dtype=np.float32)
        # raw addresses from the array interface (cheaper than .ctypes per call)
        self._check(self.lib.nedo_gpu_matvec(type_, rows, cols, w.__array_interface__["data"][0], w.nbytes,
                                             x.__array_interface__["data"][0], y.__array_interface__["data"][0]))
        return y

    def matvec_batch(self, type_: int, rows: int, cols: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        """`x.shape[0]` matvecs over one weight: y[b] = W @ x[b] (x [batch, cols])."""
        if not (isinstance(w, np.ndarray) and w.flags.c_contiguous):
            w = np.ascontiguousarray(w)
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != cols:
            raise ValueError("x must be [batch, cols]")
        y = np.empty((x.shape[0], rows), dtype=np.float32)
        self._check(self.lib.nedo_gpu_matvec_batch(type_, rows, cols, w.__array_interface__["data"][0], w.nbytes,
                                                   x.ctypes.data, y.ctypes.data, x.shape[0]))
        return y

    def embedding_row(self, type_: int, rows: int, cols: int, w: np.ndarray, row: int) -> np.ndarray:
        """nedo::kernels::embedding_row: the dequantised row (bit-exact)."""
        w = np.ascontiguousarray(w)
        out = np.empty(cols, dtype=np.float32)
        self._check(self.lib.nedo_gpu_embedding_row(type_, rows, cols, w.ctypes.data, w.nbytes, row,
                                                    out.ctypes.data))
        return out

    def weight_upload(self, w: np.ndarray) -> int:
        ptr = _vp()
        self._check(self.lib.nedo_gpu_weight_upload(w.ctypes.data, w.nbytes, ctypes.byref(ptr)))
        return ptr.value

    def weight_evict(self, w: np.ndarray) -> None:
        self._check(self.lib.nedo_gpu_weight_evict(w.ctypes.data))

    def cache_clear(self) -> None:
        self._check(self.lib.nedo_gpu_cache_clear())

    # ----------------------------------------------------- device entry points
    def matvec_dev(self, type_, rows, cols, w_ptr, x_ptr, y_ptr, batch=1, stream=0) -> None:
        self._check(self.lib.nedo_gpu_matvec_dev(type_, rows, cols, w_ptr, x_ptr, y_ptr, batch, stream))

    def reserve(self, type_, rows, cols, batch) -> None:
        """Size the buffers of a batched matvec_dev of this shape (call before graph capture)."""
        self._check(self.lib.nedo_gpu_reserve(type_, rows, cols, batch))

    def matvec_argmax_dev(self, type_, rows, cols, w_ptr, x_ptr, y_ptr, index_ptr, value_ptr=None, stream=0) -> None:
        self._check(self.lib.nedo_gpu_matvec_argmax_dev(type_, rows, cols, w_ptr, x_ptr, y_ptr, index_ptr,
                                                        value_ptr, stream))

    def argmax_dev(self, v_ptr, n, index_ptr, value_ptr=None, stream=0) -> None:
        self._check(self.lib.nedo_gpu_argmax_dev(v_ptr, n, index_ptr, value_ptr, stream))

    def argmax_dev_noalloc(self, v_ptr, n, index_ptr, value_ptr=None, stream=0) -> None:
        """argmax_dev with no allocation (a fixed device array of the library;
        overlapping calls on one device race; first call outside stream capture)."""
        self._check(self.lib.nedo_gpu_argmax_dev_noalloc(v_ptr, n, index_ptr, value_ptr, stream))

    def topk_dev(self, v_ptr, n, k, ids_ptr, vals_ptr=None, stream=0) -> None:
        """The k largest of a device fp32 vector: ids (uint32) and values, largest first."""
        self._check(self.lib.nedo_gpu_topk_dev(v_ptr, n, k, ids_ptr, vals_ptr, stream))

    def lm_head_topk(self, type_, rows, cols, w: np.ndarray, x: np.ndarray, k: int):
        """LM head (host pointers) + the top k logits: (ids uint32 [k], logits float32 [k])."""
        w = np.ascontiguousarray(w)
        x = np.ascontiguousarray(x, dtype=np.float32)
        ids = np.empty(k, dtype=np.uint32)
        vals = np.empty(k, dtype=np.float32)
        self._check(self.lib.nedo_gpu_lm_head_topk(type_, rows, cols, w.ctypes.data, w.nbytes, x.ctypes.data, k,
                                                   ids.ctypes.data, vals.ctypes.data))
        return ids, vals

    def lm_head_argmax(self, type_, rows, cols, w: np.ndarray, x: np.ndarray):
        """LM head (host pointers) + the greedy pick: (index, logit)."""
        w = np.ascontiguousarray(w)
        x = np.ascontiguousarray(x, dtype=np.float32)
        idx = ctypes.c_int64(-1)
        val = ctypes.c_float(0.0)
        self._check(self.lib.nedo_gpu_lm_head_argmax(type_, rows, cols, w.ctypes.data, w.nbytes, x.ctypes.data,
                                                     ctypes.byref(idx), ctypes.byref(val)))
        return idx.value, val.value

    def matvec_allgather_dev(self, type_, rows, cols, w_ptr, x_ptr, y_ptr, peer_y, peer_signal, row_offset,
                             stream=0) -> None:
        """This rank's rows into y_ptr, also stored on every peer (peer_y[k] + row_offset) with a
        per-CTA count on each peer's signal word."""
        n = len(peer_y)
        py = (ctypes.c_uint64 * max(n, 1))(*peer_y)
        ps = (ctypes.c_uint64 * max(n, 1))(*peer_signal)
        self._check(self.lib.nedo_gpu_matvec_allgather_dev(type_, rows, cols, w_ptr, x_ptr, y_ptr, py, ps, n,
                                                           row_offset, stream))

    def allgather_wait_dev(self, signal_ptr, expected_ptr, increment, stream=0) -> None:
        self._check(self.lib.nedo_gpu_allgather_wait_dev(signal_ptr, expected_ptr, increment, stream))

    def dequant_rows_dev(self, type_, rows, cols, w_ptr, row_begin, row_count, out_ptr, stream=0) -> None:
        self._check(self.lib.nedo_gpu_dequant_rows_dev(type_, rows, cols, w_ptr, row_begin, row_count, out_ptr,
                                                       stream))

    def status(self, stream=0) -> None:
        self._check(self.lib.nedo_gpu_status(stream))

    def plan_info(self, type_, rows, cols, batch=1) -> dict:
        out = (_u32 * 9)()
        self._check(self.lib.nedo_gpu_plan_info(type_, rows, cols, batch, out, 9))
        keys = ("path", "grid", "threads", "smem_bytes", "rows_per_tile", "slots", "slot_bytes", "warps", "launches")
        return dict(zip(keys, list(out)))


_LIB: Library | None = None


def load(path: str = LIB_PATH) -> Library:
    """The process-wide Library (loaded once)."""
    global _LIB
    if _LIB is None:
        _LIB = Library(path)
    return _LIB
