"""GGUF block formats of the matvec path, and seeded synthetic tensors.

Layouts (reference: include/nedo/gguf.hpp:18-19 type codes, src/gguf.cpp:106-114 sizes,
src/kernels.cpp:124-176 decoding):

* ``F16``  (type 1): row = ``cols`` IEEE half values, 2 bytes each.
* ``Q4_0`` (type 2): row = ``cols/32`` blocks of 18 bytes: fp16 scale ``d`` then 16 bytes;
  element ``i < 16`` is ``(byte[i] & 15) - 8``, element ``i + 16`` is ``(byte[i] >> 4) - 8``.
* ``Q8_0`` (type 8): row = ``cols/32`` blocks of 34 bytes: fp16 scale ``d`` then 32 int8.

Rows are contiguous, ``shape[0] = cols`` is the contiguous GGUF dimension.

The generators draw the distributions of the benchmark workloads with
``numpy.random.default_rng(seed)``.  fp16 scale bytes are produced once, by
numpy's round-to-nearest-even conversion, so every consumer (CPU checker and
GPU) reads identical bytes.
"""
from __future__ import annotations

import numpy as np

F16, Q4_0, Q8_0 = 1, 2, 8
TYPE_NAMES = {F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0"}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34}


def row_bytes(type_: int, cols: int) -> int:
    """Bytes of one row (src/gguf.cpp:106-114); raises on a non-multiple of 32."""
    if type_ == F16:
        return cols * 2
    if type_ in BLOCK_BYTES:
        if cols % 32:
            raise ValueError(f"{TYPE_NAMES[type_]} elements not block aligned")
        return cols // 32 * BLOCK_BYTES[type_]
    raise ValueError(f"tensor type not supported: {type_}")


def pack_q8_0(d: np.ndarray, q: np.ndarray) -> np.ndarray:
    """d: fp16 [rows, nb]; q: int8 [rows, nb, 32] -> uint8 [rows, nb*34]."""
    rows, nb = d.shape
    out = np.empty((rows, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = np.ascontiguousarray(d.astype(np.float16)).view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = q.astype(np.int8).view(np.uint8)
    return out.reshape(rows, nb * 34)


def pack_q4_0(d: np.ndarray, nib: np.ndarray) -> np.ndarray:
    """d: fp16 [rows, nb]; nib: uint8 in [0,15] [rows, nb, 32] -> uint8 [rows, nb*18]."""
    rows, nb = d.shape
    nib = nib.astype(np.uint8)
    out = np.empty((rows, nb, 18), dtype=np.uint8)
    out[:, :, 0:2] = np.ascontiguousarray(d.astype(np.float16)).view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = (nib[:, :, :16] & 15) | ((nib[:, :, 16:] & 15) << 4)
    return out.reshape(rows, nb * 18)


def dequant(type_: int, w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Vectorised dequantisation (same single fp32 multiply as src/kernels.cpp:170-176)."""
    w = np.ascontiguousarray(w).reshape(rows, row_bytes(type_, cols))
    if type_ == F16:
        return w.view(np.float16).astype(np.float32)
    nb = cols // 32
    blk = w.reshape(rows, nb, BLOCK_BYTES[type_])
    d = np.ascontiguousarray(blk[:, :, 0:2]).view(np.float16).astype(np.float32)  # [rows, nb, 1]
    if type_ == Q8_0:
        q = blk[:, :, 2:].view(np.int8).astype(np.float32)
    else:
        b = blk[:, :, 2:]
        q = np.concatenate([(b & 15).astype(np.int32) - 8, (b >> 4).astype(np.int32) - 8], axis=2).astype(np.float32)
    return (d * q).reshape(rows, cols)


def gen_weight(type_: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """Seeded weight bytes [rows, row_bytes] with the benchmark distributions:

    * Q8_0: q ~ U{-127..127}, d = fp16(|N(0, 0.02)| / 127)
    * Q4_0: nibbles ~ U{0..15}, d = fp16(|N(0, 0.02)| / 8)
    * F16 : w = fp16(N(0, 0.02))
    """
    rng = np.random.default_rng(seed)
    if type_ == F16:
        return rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32).astype(np.float16).view(np.uint8).reshape(
            rows, cols * 2)
    nb = cols // 32
    if type_ == Q8_0:
        q = rng.integers(-127, 128, size=(rows, nb, 32), dtype=np.int16).astype(np.int8)
        d = (np.abs(rng.normal(0.0, 0.02, size=(rows, nb))) / 127.0).astype(np.float32).astype(np.float16)
        return pack_q8_0(d, q)
    if type_ == Q4_0:
        nib = rng.integers(0, 16, size=(rows, nb, 32), dtype=np.uint8)
        d = (np.abs(rng.normal(0.0, 0.02, size=(rows, nb))) / 8.0).astype(np.float32).astype(np.float16)
        return pack_q4_0(d, nib)
    raise ValueError(f"tensor type not supported: {type_}")


def gen_x(cols: int, seed: int, batch: int | None = None) -> np.ndarray:
    """Seeded activations x ~ N(0, 1) fp32, shape [cols] or [batch, cols]."""
    rng = np.random.default_rng(seed + 1_000_003)
    shape = (cols,) if batch is None else (batch, cols)
    return rng.standard_normal(size=shape, dtype=np.float32)


def gen_weight_torch(torch, type_: int, rows: int, cols: int, copies: int, seed: int, device):
    """`copies` independent seeded weights ``[copies, rows * row_bytes]`` (uint8)
    generated on `device` with torch's generator, in the distributions of
    ``gen_weight`` (for sizes where numpy generation would be slow).  The bytes
    differ from ``gen_weight``'s for the same seed; a checker reads them back."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    nb = cols // 32
    if type_ == F16:
        w = (torch.randn((copies, rows, cols), generator=g, device=device) * 0.02).half()
        return w.view(torch.uint8).reshape(copies, -1)
    bb = BLOCK_BYTES[type_]
    blk = torch.empty((copies, rows, nb, bb), dtype=torch.uint8, device=device)
    if type_ == Q8_0:
        q = torch.randint(-127, 128, (copies, rows, nb, 32), generator=g, device=device, dtype=torch.int16)
        blk[..., 2:] = q.to(torch.int8).view(torch.uint8)
        d = (torch.randn((copies, rows, nb), generator=g, device=device).abs() * (0.02 / 127.0)).half()
    else:
        blk[..., 2:] = torch.randint(0, 256, (copies, rows, nb, 16), generator=g, device=device,
                                     dtype=torch.int16).to(torch.uint8)
        d = (torch.randn((copies, rows, nb), generator=g, device=device).abs() * (0.02 / 8.0)).half()
    blk[..., 0:2] = d.contiguous().view(torch.uint8).reshape(copies, rows, nb, 2)
    return blk.reshape(copies, -1)
