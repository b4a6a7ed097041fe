import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import json
    import numpy as np
    here = os.path.join(REPO, "tests", "golden")
    with open(os.path.join(here, "golden.json")) as f:
        digests = json.load(f)
    arrays = dict(np.load(os.path.join(here, "golden.npz")))
    return digests, arrays
