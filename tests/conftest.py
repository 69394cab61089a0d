"""Shared test configuration.

Markers: tests that need a CUDA device are marked `gpu` (run with `-m gpu` on a B200); the
rest run on CPU (`-m "not gpu"`). The CPU oracle (oracle/) is the checker of both.
"""

from __future__ import annotations

import itertools
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    # A GPU test on a machine without CUDA is an error in the run setup, not a skip: the
    # product path has no fallback. Without CUDA, deselect them explicitly unless -m gpu.
    pass


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run the gpu-marked tests on a B200)")
    from nanochat_filter_b200 import _lib

    _lib.load()  # fail loudly if the library was not built
    return torch.device("cuda", 0)


def load_golden(name: str) -> dict:
    """{case_key: {array_name: ndarray}} from tests/golden/<name>.npz."""
    z = np.load(os.path.join(GOLDEN, name))
    cases: dict = {}
    for k in z.files:
        case, arr = k.split("/")
        cases.setdefault(case, {})[arr] = z[k]
    return cases


def stride_layouts(shape):
    """Every dense stride layout of `shape` with optional gaps of 2 per axis (all axis orders),
    as the reference's kernel tests enumerate them (tests/ltv_scan_test_utils.py:66-77)."""
    layouts = set()
    ndim = len(shape)
    for order in itertools.permutations(range(ndim)):
        for gaps in itertools.product((1, 2), repeat=ndim):
            stride = [0] * ndim
            running = 1
            for axis, gap in zip(order, gaps):
                stride[axis] = running * gap
                running = stride[axis] * shape[axis]
            layouts.add(tuple(stride))
    return sorted(layouts)


def storage_size(shape, stride) -> int:
    return 1 + sum((s - 1) * st for s, st in zip(shape, stride))


def max_rel_err(actual, expected, floor_frac=1e-3) -> float:
    """max |a - e| / max(|e|, floor_frac * max|e|): relative error with an absolute floor so
    that entries near zero do not dominate."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    if e.size == 0:
        return 0.0
    scale = np.abs(e).max()
    if scale == 0:
        return float(np.abs(a).max())
    den = np.maximum(np.abs(e), floor_frac * scale)
    return float((np.abs(a - e) / den).max())


def max_rel_err_rms(actual, expected) -> float:
    """max |a - e| / max(|e|, rms(e)): relative error with the absolute floor at the tensor's RMS
    (the form of the reference's own kernel tests, |a - e| <= atol + rtol |e| with atol = rtol on
    unit-scale data). A bf16 value that rounds to the neighbouring value in one implementation and
    not in the other (fp32 vs float64 accumulation of a GEMM) moves every later state of the scan by
    a fraction of that value's ulp; relative to entries far below the tensor's scale that is not
    small, so the floor sits at the scale of the data."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    if e.size == 0:
        return 0.0
    rms = float(np.sqrt(np.mean(e * e)))
    if rms == 0:
        return float(np.abs(a).max())
    return float((np.abs(a - e) / np.maximum(np.abs(e), rms)).max())


def assert_allclose_np(actual, expected, rtol, atol, label=""):
    a = np.asarray(actual, dtype=np.float32)
    e = np.asarray(expected, dtype=np.float32)
    np.testing.assert_allclose(a, e, rtol=rtol, atol=atol, err_msg=label)
