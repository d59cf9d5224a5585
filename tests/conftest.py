import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)
TESTS = os.path.join(REPO, "tests")
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_golden(name: str) -> dict:
    """Loads tests/golden/<name>.npz; tensors come back with their stored dtype."""
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    out = {}
    for k in z.files:
        if k.endswith("__dtype"):
            continue
        a = z[k]
        dt = str(z[k + "__dtype"]) if (k + "__dtype") in z.files else None
        if dt is None:
            out[k] = a.item() if a.shape == () else a
            continue
        t = torch.from_numpy(a.copy())
        if dt == "bfloat16":
            t = t.view(torch.bfloat16)
        out[k] = t
    return out


def golden_names(prefix: str) -> list[str]:
    return sorted(f[:-4] for f in os.listdir(GOLDEN) if f.startswith(prefix) and f.endswith(".npz"))


@pytest.fixture(scope="session")
def cuda_dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
