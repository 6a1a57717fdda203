import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")


@pytest.fixture(scope="session")
def plan_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("plans"))


@pytest.fixture(scope="session")
def model_plans(plan_dir):
    from infvino_b200 import plangen
    return {name: fn(os.path.join(plan_dir, name)) for name, fn in plangen.MODELS.items()}
