import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


def golden_cases(golden, prefix="v/"):
    """Group golden keys 'v/<dtype>/<pack>/<MxN>/<sp>/<field>' by case."""
    cases = {}
    for k, v in golden.items():
        if not k.startswith(prefix):
            continue
        case, field = k.rsplit("/", 1)
        cases.setdefault(case, {})[field] = v
    return cases


def parse_case(case):
    _, dtype, pack, shape, sp = case.split("/")
    M, N = (int(s) for s in shape.split("x"))
    return dtype, bool(int(pack)), (M, N), float(sp)
