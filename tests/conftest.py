"""Shared pytest configuration.

* registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``);
* puts the repository root (``oracle``) and the package directory
  (``itmo-final-project_b200``, home of ``int4_b200``) on ``sys.path``;
* loads the committed golden fixtures once per session.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "itmo-final-project_b200")
GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG_DIR, GOLDEN_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def golden_meta():
    with open(os.path.join(GOLDEN_DIR, "golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def golden_arrays():
    with np.load(os.path.join(GOLDEN_DIR, "golden_small.npz")) as d:
        return {k: d[k] for k in d.files}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"kernels are built for sm_100a, found sm_{major}{minor}"
    return torch.device("cuda", 0)
