"""Shared test set-up: the `gpu` marker, import paths, and fixtures for the library and checkers.

CPU tests (`-m "not gpu"`) cover the oracle against the reference and its golden vectors, the host
logic and the C ABI surface. GPU tests (`-m gpu`) are the parity tests proper: they call the CUDA
kernels through the C ABI and compare with the oracle and with the reference's own CUDA kernels.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("bare-metal-gpt2_b200", "oracle", ""):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

import oracle as O  # noqa: E402  (test infrastructure)

# Parity bar from the task statement: fp16 storage, fp32 accumulation.
ABS_TOL = 2e-3   # max |gpu - ref| over all elements
REL_TOL = 1e-2   # max |gpu - ref| / max |ref|  (the reference's rel_err, bench/correctness_cuda.cu:70-75)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def assert_close(got: np.ndarray, ref: np.ndarray, what: str, abs_tol: float = ABS_TOL,
                 rel_tol: float = REL_TOL) -> None:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} vs {ref.shape}"
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = np.abs(got - ref)
    max_abs = float(err.max()) if err.size else 0.0
    rel = max_abs / (float(np.abs(ref).max()) + 1e-9) if err.size else 0.0
    assert max_abs <= abs_tol and rel <= rel_tol, (
        f"{what}: max_abs={max_abs:.3e} (tol {abs_tol}) rel={rel:.3e} (tol {rel_tol}) at "
        f"{np.unravel_index(int(err.argmax()), err.shape)}")


@pytest.fixture(scope="session")
def oracle():
    return O.Oracle()


@pytest.fixture(scope="session")
def lib():
    import gpt2_b200
    return gpt2_b200.load()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    torch.cuda.init()
    return torch


@pytest.fixture(scope="session")
def ref_gpu():
    return O.RefGPU()
