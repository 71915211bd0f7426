"""Reader for tests/golden/golden_cases.npz (written by tests/golden/make_golden.py
from the reference implementation run on CPU)."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_cases.npz")


def load_cases():
    z = np.load(GOLDEN)
    meta = json.loads(bytes(z["__meta__"]).decode())
    cases = []
    for m in meta:
        n = m["name"]
        arrays = {key.split("/", 1)[1]: z[key] for key in z.files if key.startswith(n + "/")}
        cases.append((m, arrays))
    return cases
