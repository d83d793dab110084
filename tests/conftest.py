import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; the parity tests proper")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden():
    import json
    with open(os.path.join(GOLDEN, "sdpa_golden.json")) as f:
        index = json.load(f)["cases"]
    z = np.load(os.path.join(GOLDEN, "sdpa_golden.npz"))
    cases = []
    for meta in index:
        name = meta["name"]
        arrays = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
        cases.append((meta, arrays))
    return cases


def rel_err(got, ref):
    """max|got - ref| / max|ref| (the north star's tolerance measure)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.max(np.abs(ref)) if ref.size else 0.0
    if ref.size == 0:
        return 0.0
    return float(np.max(np.abs(got - ref)) / (scale if scale > 0 else 1.0))
