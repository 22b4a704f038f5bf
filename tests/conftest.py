"""Shared test setup: import paths, the `gpu` marker, golden-fixture helpers.

`-m "not gpu"` runs everything that needs no GPU (the oracle against the
reference's golden vectors, host-side bookkeeping, the C ABI surface, the
multi-rank host logic over gloo).  `-m gpu` runs the parity tests proper:
the CUDA kernels through the C ABI against the oracle and the golden vectors.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "llm-inference-scheduler_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG_ROOT, os.path.join(ROOT, "oracle"), GOLDEN, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

# Tolerances.  Product vs oracle: the north-star bounds (1e-5 fp32, 2e-3 fp16);
# bf16 has 8x coarser rounding than fp16, so 8x the fp16 bound.
PRODUCT_ATOL = {"f32": 1e-5, "f16": 2e-3, "bf16": 1.6e-2}
# Oracle vs the reference's golden vectors: about one ulp of the output dtype.
ORACLE_ATOL = {"f32": 2e-6, "f16": 1e-3, "bf16": 4e-3}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name))


def as_f32(a: np.ndarray, dt: str) -> np.ndarray:
    import cases

    return cases.to_float32(a, dt)


def max_abs_diff(a, b, dt: str) -> float:
    return float(np.max(np.abs(as_f32(a, dt) - as_f32(b, dt)))) if a.size else 0.0


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    oracle.lib()
    return oracle
