"""Shared fixtures for the parity suite.

Markers:
  gpu  -- needs a CUDA device (B200); everything else runs on CPU.

Layout the tests rely on:
  oracle/          CPU checkers (C restatement + the reference compiled from source)
  nedo.cpp_b200/   the product: lib/libnedo_gpu.so and its Python binding nedo_gpu
  tests/golden/    fixtures produced by the reference itself
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "nedo.cpp_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "matvec_golden.npz")

# Tolerance contract of the matvec path: per output element
#   |y_gpu - y_ref| <= TOL * sum_i |w_i * x_i|     (w_i dequantised)
TOL = 1e-4


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O

    O.build()
    return O.Oracle()


@pytest.fixture(scope="session")
def reference():
    import oracle as O

    if not O.Reference.available():
        pytest.skip("the reference was not compiled here (oracle/_ref absent)")
    return O.Reference()


@pytest.fixture(scope="session")
def golden():
    data = np.load(GOLDEN)
    cases = {}
    for name in data["names"]:
        name = str(name)
        t, rows, cols = (int(v) for v in data[f"{name}/meta"])
        cases[name] = dict(
            type=t, rows=rows, cols=cols, w=data[f"{name}/w"], x=data[f"{name}/x"],
            y_native=data[f"{name}/y_native"], y_portable=data[f"{name}/y_portable"],
            deq_rows=data[f"{name}/deq_rows"], deq=data[f"{name}/deq"], absdot=data[f"{name}/absdot"])
    return cases


@pytest.fixture(scope="session")
def lib():
    import nedo_gpu

    return nedo_gpu.load()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def assert_within_tol(y, y_ref, absdot, tol=TOL, what=""):
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    err = np.abs(y - y_ref)
    bound = tol * np.asarray(absdot, dtype=np.float64)
    bad = np.nonzero(~(err <= bound))[0]
    if bad.size:
        i = bad[np.argmax(err[bad] / np.maximum(bound[bad], 1e-300))]
        raise AssertionError(
            f"{what}: {bad.size}/{y.size} outputs outside {tol}*sum|w*x|; worst row {i}: "
            f"gpu={y[i]!r} ref={y_ref[i]!r} err={err[i]:.3e} bound={bound[i]:.3e}")
