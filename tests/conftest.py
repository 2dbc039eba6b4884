import importlib
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PACKAGE = "latentpagedattention-rs_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


def load_package():
    return importlib.import_module(PACKAGE)


def load_ops():
    return importlib.import_module(PACKAGE + ".ops")


def load_golden_json(name: str) -> dict:
    with open(os.path.join(GOLDEN, name), encoding="utf-8") as f:
        return json.load(f)


def load_reference_fixture(name: str) -> dict:
    return load_golden_json(os.path.join("reference", name))


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def ops():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return load_ops()
