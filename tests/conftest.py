"""Shared pytest setup: the ``gpu`` marker, import paths and fixtures."""

import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_NAME = "care-kv-sparse-residual-correction-for-low-bit-kv-cache-quantization_b200"
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built sm_100a library")


def load_pkg():
    """Import the product package (its directory name is not an identifier)."""
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def carekv():
    return load_pkg()


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
