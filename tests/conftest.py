"""Shared pytest setup: markers, import paths for the product binding and the oracle."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "llm-accel_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: CPU test that takes tens of seconds")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    O.set_exp_mode(O.EXP_TRUNC)
    return O


@pytest.fixture(scope="session")
def llmx():
    import llmx as X
    X.lib()
    return X
