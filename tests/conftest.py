"""Pytest configuration: the `gpu` marker, per-test seeding, library build.

Seeding follows the reference's tests/conftest.py:8-37: every module and test
reseeds `random` and `torch` with sha256(test path) mod 2**32, so inputs are
deterministic per test id.
"""

import hashlib
import random
import shutil

import pytest
import torch


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")
    # Build the in-tree libraries when sources are newer (nvcc cross-compiles
    # without a GPU; gcc builds the CPU oracle).
    from ninetoothed_b200 import _build

    if shutil.which("nvcc") or _build.LIBRARY.is_file():
        if _build.is_stale() and shutil.which("nvcc"):
            _build.build()
    import oracle

    oracle.build()


def _hash(string):
    return int(hashlib.sha256(string.encode("utf-8")).hexdigest(), 16) % 2**32


def _set_random_seed(seed):
    random.seed(seed)
    torch.manual_seed(seed)


@pytest.fixture(autouse=True)
def set_seed_per_test(request):
    _set_random_seed(_hash(f"{request.module.__name__.replace('.', '/')}.py::{request.node.name}"))


def pytest_collection_modifyitems(config, items):
    del config
    if torch.cuda.is_available() and torch.cuda.get_device_capability() >= (10, 0):
        return
    skip = pytest.mark.skip(reason="needs an sm_100 GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
