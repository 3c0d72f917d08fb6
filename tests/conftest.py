import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402

__graft_entry__.import_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) CUDA device")


@pytest.fixture(scope="session")
def golden():
    """{case name: {field: array}} from tests/golden/attention_golden.npz (reference outputs)."""
    import numpy as np

    data = np.load(os.path.join(ROOT, "tests", "golden", "attention_golden.npz"))
    cases = {}
    for key in data.files:
        name, field = key.split("/")
        cases.setdefault(name, {})[field] = data[key]
    return cases
