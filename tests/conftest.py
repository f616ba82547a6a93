import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: large model sizes (minutes)")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Build the oracle (gcc) and the synthetic-model generator once per session."""
    import oracle
    from talos_b200 import build

    oracle.build()
    build.build_synth()
