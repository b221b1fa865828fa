import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "metal-infer-rs_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

# Streams of the synthetic inputs (weights use (layer + 1) * 16 + role).
INPUT_STREAM = 1 << 20


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def ctx():
    import metal_infer as mi
    return mi.MetalContext(0)
