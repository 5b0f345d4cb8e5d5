"""Test configuration.

Markers:
  gpu   needs a CUDA device (run with `-m gpu`); everything else runs on CPU.

The package lives in mhc-proj_b200/ (import name `mhc_proj`); the oracle
(test infrastructure) in oracle/.  Both directories go on sys.path here.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "mhc-proj_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def golden_cases():
    return sorted(f[len("golden_"):-len(".npz")] for f in os.listdir(GOLDEN)
                  if f.startswith("golden_") and f.endswith(".npz"))


def load_golden(name):
    import numpy as np

    return dict(np.load(os.path.join(GOLDEN, f"golden_{name}.npz")))
