import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def load_cases(path, prefix="c"):
    """Unflatten a golden npz written as <prefix><i>_<key> arrays."""
    import numpy as np

    z = np.load(path, allow_pickle=False)
    n = int(z["n_cases"])
    cases = []
    for i in range(n):
        pre = f"{prefix}{i}_"
        cases.append({k[len(pre):]: z[k] for k in z.files if k.startswith(pre)})
    return cases, z
