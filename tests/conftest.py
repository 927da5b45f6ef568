import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the CUDA kernels")


@pytest.fixture(scope="session")
def mini_models():
    from tests.synth import presets

    return {name: presets.model_path(name) for name in presets.CONFIGS if name.startswith("mini_")}
