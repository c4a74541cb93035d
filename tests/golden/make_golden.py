"""Regenerate tests/golden/matvec_golden.npz from the reference itself.

Runs the reference's own src/kernels.cpp (compiled from source by oracle/Makefile
into oracle/_ref/, both the AVX2/FMA "native" flavour and the scalar "portable"
flavour) on seeded inputs and stores inputs and outputs.  The fixtures travel
with the repository, so the parity tests can pin both the C restatement and the
CUDA kernels to the reference where the reference sources are absent.

Cases:
  * the reference's own known-answer tests (tests/test_kernels.cpp:33-65)
  * seeded matrices of every type at small shapes, including ragged row counts,
    an odd block count (generic kernel path) and column counts of the
    benchmark workloads (1536, 2048, 4096)

Usage:  make -C oracle all && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "nedo.cpp_b200"))

from oracle import REF_LIB, REF_PORTABLE_LIB, Oracle, Reference  # noqa: E402
from nedo_gpu import blocks as B  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "matvec_golden.npz")


def kat_cases():
    one = np.array([1.0], dtype=np.float32).astype(np.float16).view(np.uint8)
    q8 = np.zeros(34, dtype=np.uint8)
    q8[0:2] = one
    q8[2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    q4 = np.zeros(18, dtype=np.uint8)
    q4[0:2] = one
    q4[2:] = np.array([((15 - i) << 4) | i for i in range(16)], dtype=np.uint8)
    ones = np.ones(32, dtype=np.float32)
    return [("kat_q8", B.Q8_0, 1, 32, q8, ones), ("kat_q4", B.Q4_0, 1, 32, q4, ones)]


def seeded_cases():
    shapes = {
        B.Q8_0: [(40, 512), (7, 1536), (33, 96), (24, 4096), (130, 2048)],
        B.Q4_0: [(40, 512), (7, 1536), (33, 96), (24, 4096), (130, 2048)],
        B.F16: [(40, 512), (7, 1536), (33, 104), (16, 2048), (9, 4096)],
    }
    out = []
    seed = 100
    for t, lst in shapes.items():
        for rows, cols in lst:
            seed += 1
            w = B.gen_weight(t, rows, cols, seed)
            x = B.gen_x(cols, seed)
            out.append((f"{B.TYPE_NAMES[t].lower()}_{rows}x{cols}", t, rows, cols, w.reshape(-1), x))
    return out


def main() -> None:
    if not (os.path.exists(REF_LIB) and os.path.exists(REF_PORTABLE_LIB)):
        sys.exit("oracle/_ref is not built: run `make -C oracle all` where the reference sources exist")
    ref, ref_p, orc = Reference(REF_LIB), Reference(REF_PORTABLE_LIB), Oracle()
    data = {}
    names = []
    for name, t, rows, cols, w, x in kat_cases() + seeded_cases():
        w = np.ascontiguousarray(w, dtype=np.uint8)
        names.append(name)
        data[f"{name}/meta"] = np.array([t, rows, cols], dtype=np.int64)
        data[f"{name}/w"] = w
        data[f"{name}/x"] = x
        data[f"{name}/y_native"] = ref.matvec(t, rows, cols, w, x)
        data[f"{name}/y_portable"] = ref_p.matvec(t, rows, cols, w, x)
        deq_rows = sorted({0, rows // 2, rows - 1})
        data[f"{name}/deq_rows"] = np.array(deq_rows, dtype=np.int64)
        data[f"{name}/deq"] = np.stack([ref.embedding_row(t, rows, cols, w, r) for r in deq_rows])
        data[f"{name}/absdot"] = orc.abs_dot(t, rows, cols, w, x)
    data["names"] = np.array(names)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT}: {len(names)} cases, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
