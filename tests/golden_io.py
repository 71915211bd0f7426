"""Readers for tests/golden/golden_cases.npz and golden_bwd.npz (written by
tests/golden/make_golden.py and make_golden_bwd.py from the reference
implementation run on CPU)."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_cases.npz")
GOLDEN_BWD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_bwd.npz")


def load_cases(path=GOLDEN):
    z = np.load(path)
    meta = json.loads(bytes(z["__meta__"]).decode())
    cases = []
    for m in meta:
        n = m["name"]
        arrays = {key.split("/", 1)[1]: z[key] for key in z.files if key.startswith(n + "/")}
        cases.append((m, arrays))
    return cases


def load_bwd_cases():
    return load_cases(GOLDEN_BWD)
