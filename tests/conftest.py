"""Shared pytest set-up: the `gpu` marker, the package loader and fixtures."""

from __future__ import annotations

import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu on the GPU box")


@pytest.fixture(scope="session")
def golden() -> dict:
    with open(os.path.join(GOLDEN, "golden.json")) as fh:
        return json.load(fh)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def pkg():
    """The CUDA package (llm-kv260_b200), loaded the way bench.py loads it."""
    import __graft_entry__
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def cuda_lib(pkg):
    """The loaded C-ABI library on a GPU box; the GPU tests depend on it.
    A GPU test without a GPU fails: there is no CPU path to fall back to."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a -m gpu test ran without a CUDA device")
    return pkg.lib()
