import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def rel_err(actual, expected):
    """max |a - e| / max |e|  (the relative tolerance used for features)."""
    import numpy as np
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return float(np.abs(a - e).max() / max(np.abs(e).max(), 1e-30))


def carrier_mismatches(got_idx, ref_idx, ref_center, center_tol=1e-3):
    """Images whose carriers differ from the reference.

    The carrier SET must match exactly.  The ORDER is ascending centre of mass
    (model.py:1169-1171, an unstable argsort over float32 centres); two
    carriers whose centres agree to ``center_tol`` (16 ulp at the largest
    28x28 centre) have no reproducible order, so only such pairs may swap.
    Returns [(image, "set" | "order")].
    """
    import numpy as np
    got_idx = np.asarray(got_idx)
    ref_idx = np.asarray(ref_idx)
    centers = np.asarray(ref_center)[:, 1:]
    out = []
    for b in range(ref_idx.shape[0]):
        if np.array_equal(got_idx[b], ref_idx[b]):
            continue
        if set(got_idx[b].tolist()) != set(ref_idx[b].tolist()):
            out.append((b, "set"))
        elif np.abs(centers[b][got_idx[b]] - centers[b][ref_idx[b]]).max() > center_tol:
            out.append((b, "order"))
    return out
