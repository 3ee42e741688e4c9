import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
GOLDEN_CASES = ("k4_h256_i128", "k8_h384_i128")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on the B200 box)")


def load_golden(name: str) -> dict:
    z = np.load(GOLDEN_DIR / f"{name}.npz")
    return {k: z[k] for k in z.files}


def golden_groups(gold: dict) -> list[dict]:
    """Slot tensor dicts (on-disk suffix -> array) of a golden case."""
    h, i, e, k = (int(v) for v in gold["meta"][:4])
    groups = []
    for g in range(e // k):
        pre = f"g{g}."
        groups.append({kk[len(pre):]: v for kk, v in gold.items() if kk.startswith(pre)})
    return groups


@pytest.fixture(params=GOLDEN_CASES)
def golden(request):
    return load_golden(request.param)
