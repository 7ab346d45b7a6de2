"""Shared fixtures.  Tests marked ``gpu`` need an sm_100 device; the rest run on CPU."""
from __future__ import annotations

import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"

# Parity tolerances (include/p100/tolerance.h:20-31; tests/h2_mmv_gpu.cu:89):
QMV_NORM_TOL = 1e-3          # |y_gpu - y_q81| <= 1e-3 * ||w|| * ||x||
OUT_ABS_TOL, OUT_REL_TOL, LSE_ABS_TOL = 1e-3, 2e-3, 1e-3
ATTN_MAX_REL_TOL = 1e-3      # max|O - O_ref| / max|O_ref| (tests/error_budget.cpp:78)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")
    config.addinivalue_line("markers", "multigpu: needs two or more sm_100 GPUs")


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.Ref.available():
        pytest.skip("oracle/_ref (the reference compiled from its sources) is not built here")
    return oracle.Ref()


@pytest.fixture(scope="session")
def lib():
    import p100_b200
    return p100_b200.lib()


@pytest.fixture(scope="session")
def cuda():
    """torch with a usable sm_100 device; GPU tests fail loudly without one."""
    import torch
    import p100_b200
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    status = p100_b200.device_check(0)
    assert status == 0, f"device 0 is not usable by the library: {p100_b200.last_error()}"
    return torch


def out_within_tolerance(got, ref):
    """tolerance.h:24-26 element-wise."""
    return np.abs(got.astype(np.float64) - ref) <= OUT_ABS_TOL + OUT_REL_TOL * np.abs(ref)


def lse_within_tolerance(got, ref):
    """tolerance.h:28-31 element-wise (-inf must stay -inf)."""
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    neg = np.isneginf(ref)
    with np.errstate(invalid="ignore"):
        ok = np.where(neg, np.isneginf(got), np.abs(got - ref) <= LSE_ABS_TOL)
    return ok


def golden(name):
    return np.load(GOLDEN / name)
