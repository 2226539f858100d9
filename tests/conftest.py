import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "lastro-rust_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); parity tests through the C ABI")


@pytest.fixture(scope="session")
def pool():
    import oracle as O
    p = O.Pool(min(8, os.cpu_count() or 1))
    yield p
    p.close()


@pytest.fixture(scope="session")
def gpu_ctx():
    import lastro_b200 as LB
    ctx = LB.Context(0)
    yield ctx
    ctx.close()
