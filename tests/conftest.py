import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    return oracle


@pytest.fixture(scope="session")
def rtlib():
    import rich_triplet_b200 as rt
    return rt.lib()


@pytest.fixture(scope="session")
def gpu_ctx():
    from rich_triplet_b200.ops import Context
    ctx = Context(0)
    yield ctx
    ctx.close()
