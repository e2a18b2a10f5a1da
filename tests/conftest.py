"""Shared pytest setup: the `gpu` marker, import paths and oracle fixtures."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "seedvr2-ncnn-valkan_b200"), os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def port():
    import oracle
    if not os.path.exists(oracle.PORT_SO):
        oracle.build()
    return oracle.port()


@pytest.fixture(scope="session")
def ref():
    import oracle
    r = oracle.ref()
    if r is None:
        pytest.skip("reference build oracle/_ref/libs2ref.so not present")
    return r


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))
    return load


def from_bf16_bits(u: np.ndarray) -> np.ndarray:
    return (np.asarray(u, np.uint32) << 16).view(np.float32)
