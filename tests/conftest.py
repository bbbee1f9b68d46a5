import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.join(ROOT, "tests")
GOLDEN = os.path.join(TESTS, "golden")
for p in (ROOT, TESTS, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def golden_names():
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))


def load_golden(name):
    """(recipe dict, expected outputs dict) of one golden fixture."""
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    recipe = json.loads(str(z["recipe"]))
    return recipe, {k: z[k] for k in z.files if k != "recipe"}


@pytest.fixture(scope="session")
def golden():
    return load_golden
