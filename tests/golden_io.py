"""Loader for the JSON golden fixtures written by tests/golden/make_golden.py."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _arr(t):
    dt = np.dtype(t["dtype"])
    if dt == np.float32:
        a = np.array(t["data"], dtype=np.uint32).view(np.float32)
    else:
        a = np.array(t["data"], dtype=np.int64).astype(dt)
    return a.reshape(t["shape"])


def load(case):
    with open(os.path.join(GOLDEN, case + ".json")) as f:
        e = json.load(f)
    return [_arr(t) for t in e["inputs"]], [_arr(t) for t in e["outputs"]]


def attributes(case):
    """Scalar node attributes recorded with the fixture (may be empty)."""
    with open(os.path.join(GOLDEN, case + ".json")) as f:
        return json.load(f).get("attributes", {})
