import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
for sub in ("decision-programs_b200", "oracle", "tests"):
    p = str(ROOT / sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def dp():
    import dp_gbdt
    dp_gbdt.lib()
    return dp_gbdt


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.lib()
    return oracle
