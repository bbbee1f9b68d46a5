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


def pytest_terminal_summary(terminalreporter):
    """The largest per-element relative error (floor: parity.ELEM_FLOOR x
    max|ref|) and max-normalised error of each compared quantity."""
    try:
        from parity import ELEM_FLOOR, ELEM_REPORT
    except ImportError:
        return
    if not ELEM_REPORT:
        return
    terminalreporter.section("parity: largest errors per compared quantity")
    terminalreporter.write_line(f"{'quantity':32s} {'per-element':>12s} {'max-normalised':>15s}  "
                                f"(per-element floor {ELEM_FLOOR:g} x max|ref|)")
    for k, (ee, e) in sorted(ELEM_REPORT.items()):
        terminalreporter.write_line(f"{k[:32]:32s} {ee:12.3e} {e:15.3e}")
