"""The persistent forward kernel (one CTA per SM taking query tiles from a
work counter) against the one-tile-per-CTA kernel: the kernel is chosen once
per process (TDA_B200_FWD_PERSISTENT), so each is run in a child process on
the same seeded inputs and the outputs must be bit-identical -- both run the
same per-tile arithmetic, only the scheduling differs."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

# op, (B, H, S, D), beta, lambda, p, normalize, out_f32
CASES = [
    ("rect", (2, 3, 1000, 128), 1.0, 0.0, 2.0, True, False),
    ("rect", (1, 4, 300, 64), 0.5, 0.0, 3.0, True, False),
    ("rect", (1, 2, 520, 128), -0.5, 0.0, 2.0, True, False),
    ("rect", (1, 2, 384, 128), 1.0, 0.0, 1.5, False, True),
    ("diff", (1, 3, 700, 128), 1.0, 0.5, 2.0, True, False),
    ("diff", (2, 2, 200, 64), -0.7, 0.3, 2.0, True, True),
    ("diff", (1, 2, 256, 128), 1.0, 0.8, 1.0, False, False),
]

CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
import tda_b200
cases = eval(sys.argv[2])
out = {}
for i, (op, shape, beta, lam, p, norm, f32) in enumerate(cases):
    g = torch.Generator(device="cpu").manual_seed(100 + i)
    xs = [torch.randn(shape, generator=g).to(torch.bfloat16).cuda() for _ in range(5)]
    od = torch.float32 if f32 else None
    if op == "rect":
        o = tda_b200.rect_forward(xs[0], xs[1], xs[2], beta, p, norm, out_dtype=od)
    else:
        o = tda_b200.diff_forward(*xs, beta, lam, p, norm, out_dtype=od)
    tda_b200.check_status()
    out[f"c{i}"] = o.float().cpu().numpy()
np.savez(sys.argv[3], **out)
"""


def _run(mode, path):
    env = dict(os.environ, TDA_B200_FWD_PERSISTENT=mode)
    subprocess.run([sys.executable, "-c", CHILD, ROOT, repr(CASES), path], env=env, check=True, timeout=600)
    return np.load(path)


def test_persistent_kernel_matches_per_tile_kernel(tmp_path):
    a = _run("1", str(tmp_path / "persistent.npz"))
    b = _run("0", str(tmp_path / "per_tile.npz"))
    for i in range(len(CASES)):
        assert np.array_equal(a[f"c{i}"], b[f"c{i}"]), CASES[i]
        assert np.isfinite(a[f"c{i}"]).all()
