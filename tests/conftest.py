import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


@pytest.fixture(autouse=True)
def _reset_comm():
    from neural_scaling_weather_b200.parallel import comm
    from neural_scaling_weather_b200.ops import weights

    yield
    comm.reset()
    weights.clear()
    from neural_scaling_weather_b200.parallel import symm

    symm.reset()
    from neural_scaling_weather_b200.parallel import halo

    halo.reset()
