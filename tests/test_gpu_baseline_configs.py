"""Parity at the full shapes of BASELINE configs 2, 3 and 4 (and dense / beta < 0
variants of config 3), through the public API, against the fp64 oracle.

The whole problem runs on the GPU at its real size, so every scheduling path
the bench uses is exercised: up to 64 (S = 8192) and 256 (S = 32768) key tiles
per query tile, the grouped longest-first launch order over all (batch, head)
slices, the key-table zero-half test at large tau (beta = 1.5), the persistent
kernel, and the O accumulation over a whole 32768-key row.  The oracle then
recomputes a sample: three (batch, head) slices (the first, the last and one
seeded) and, in each, 256 query rows (the first 64, the last 64 and 128 spread
over the sequence).

Each kernel schedule runs in a child process, because the forward kernel
(one CTA per query tile, the persistent one-CTA-per-SM kernel, or the
CTA-pair kernel) is chosen once per process (TDA_B200_FWD_PERSISTENT,
TDA_B200_FWD_PAIR).

Tolerances, as for every bf16 parity test here (rel-L2 over the sampled rows):
  * the kernel's fp32 accumulator output vs the oracle:   <= 1e-3
  * the public bf16 output vs the bf16-rounded oracle:     <= 1e-3
(rounding the exact result to bf16 alone is ~1.7e-3 rel-L2, so the bf16
output is compared with the rounded oracle).

Reference: triton_threshold_attention.py:62-109 (the full-S loop with
tau = beta * sqrt(2 log(i + 1) / D)) and :489-519 (the differential form).
"""
import os
import subprocess
import sys
import zlib

import numpy as np
import pytest

from oracle import tda_oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
TOL = 1e-3

# name: (op, (B, H, S, D), beta, lambda, p, normalize)
CONFIGS = {
    "cfg2_rect_4x32x4096": ("rect", (4, 32, 4096, 128), 1.0, 0.0, 2.0, True),
    "cfg3_diff_8x32x8192": ("diff", (8, 32, 8192, 128), 1.0, 0.5, 2.0, True),
    "cfg3_rect_8x32x8192": ("rect", (8, 32, 8192, 128), 1.0, 0.0, 2.0, True),
    "cfg4_diff_1x16x32768": ("diff", (1, 16, 32768, 128), 1.5, 0.8, 2.0, True),
    # every causal tile processed with dense P (beta = 0), and every tile of
    # the row processed, masked entries included (beta < 0)
    "cfg3_diff_dense_beta0": ("diff", (8, 32, 8192, 128), 0.0, 0.5, 2.0, True),
    "cfg3_diff_beta_neg": ("diff", (8, 32, 8192, 128), -0.5, 0.5, 2.0, True),
    "s8k_rect_beta_neg_p3": ("rect", (2, 8, 8192, 128), -0.5, 0.0, 3.0, True),
}

CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
import tda_b200
from test_gpu_baseline_configs import CONFIGS, make_inputs, sample_of
names = sys.argv[2].split(",")
res = {}
for name in names:
    op, shape, beta, lam, p, norm = CONFIGS[name]
    xs = make_inputs(name)
    bhs, rows = sample_of(name)
    if op == "diff":
        acc = tda_b200.diff_forward(*xs, beta, lam, p, norm, out_dtype=torch.float32)
        out = tda_b200.differential_threshold_rela_triton(*xs, torch.tensor(beta), torch.tensor(lam), p, norm)
    else:
        acc = tda_b200.rect_forward(xs[0], xs[1], xs[2], beta, p, norm, out_dtype=torch.float32)
        out = tda_b200.threshold_rela_triton(xs[0], xs[1], xs[2], torch.tensor(beta), p, norm)
    tda_b200.check_status()
    B, H, S, D = shape
    r = torch.as_tensor(rows, device=acc.device)
    a = acc.view(B * H, S, D)[bhs][:, r].float().cpu().numpy()
    o = out.view(B * H, S, D)[bhs][:, r].float().cpu().numpy()
    assert out.dtype == torch.bfloat16 and tuple(out.shape) == shape
    res[name + "/acc"] = a
    res[name + "/out"] = o
    del xs, acc, out
    torch.cuda.empty_cache()
np.savez(sys.argv[3], **res)
"""


def _n_inputs(op):
    return 5 if op == "diff" else 3


def make_inputs(name, bhs=None):
    """Seeded N(0,1) bf16 inputs of a config on cuda:0, one generator per
    (tensor, flattened head), so a sampled head can be regenerated alone.
    Returns full (B, H, S, D) tensors, or (len(bhs), S, D) tensors of the
    listed heads when ``bhs`` is given."""
    import torch
    op, (B, H, S, D), *_ = CONFIGS[name]
    heads = list(range(B * H)) if bhs is None else list(bhs)
    xs = []
    for t in range(_n_inputs(op)):
        x = torch.empty((len(heads), S, D), dtype=torch.bfloat16, device="cuda")
        for i, bh in enumerate(heads):
            g = torch.Generator(device="cuda").manual_seed(7_000_003 * (t + 1) + bh)
            x[i] = torch.randn((S, D), generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)
        xs.append(x.view(B, H, S, D) if bhs is None else x)
    return xs


def sample_of(name):
    """(batch, head) slices and query rows checked against the oracle."""
    op, (B, H, S, D), *_ = CONFIGS[name]
    rng = np.random.Generator(np.random.PCG64(zlib.crc32(name.encode())))
    seeded = int(rng.integers(1, B * H - 1)) if B * H > 2 else 0
    bhs = sorted({0, B * H - 1, seeded})
    spread = rng.choice(np.arange(64, S - 64), size=128, replace=False)
    rows = np.unique(np.concatenate([np.arange(64), np.arange(S - 64, S), spread]))
    return bhs, rows


def _oracle(name, bhs, rows):
    """fp64 oracle on the sampled heads / rows: (len(bhs), len(rows), D)."""
    op, (B, H, S, D), beta, lam, p, norm = CONFIGS[name]
    xs = make_inputs(name, bhs)
    ref = []
    for i in range(len(bhs)):
        a = [x[i].float().cpu().numpy()[None, None] for x in xs]
        if op == "diff":
            r = O.diff_fwd(*a, beta, lam, p, norm, rows=rows)
        else:
            r = O.rect_fwd(*a, beta, p, norm, rows=rows)
        ref.append(r[0, 0, rows])
    return np.stack(ref)


SCHEDULES = {
    "per_tile": {"TDA_B200_FWD_PERSISTENT": "0", "TDA_B200_FWD_PAIR": "0"},
    "persistent": {"TDA_B200_FWD_PERSISTENT": "1", "TDA_B200_FWD_PAIR": "0"},
    "pair": {"TDA_B200_FWD_PERSISTENT": "0", "TDA_B200_FWD_PAIR": "1"},
}


@pytest.fixture(scope="module", params=list(SCHEDULES))
def gpu_results(request, tmp_path_factory):
    path = str(tmp_path_factory.mktemp("cfg") / f"{request.param}.npz")
    env = dict(os.environ, **SCHEDULES[request.param])
    subprocess.run([sys.executable, "-c", CHILD, ROOT, ",".join(CONFIGS), path], env=env, check=True,
                   timeout=1200)
    return np.load(path)


_REFS = {}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_full_shape_config_against_oracle(gpu_results, name):
    bhs, rows = sample_of(name)
    if name not in _REFS:
        _REFS[name] = _oracle(name, bhs, rows)
    ref = _REFS[name]
    acc = gpu_results[name + "/acc"]
    out = gpu_results[name + "/out"]
    assert acc.shape == ref.shape and np.isfinite(acc).all() and np.isfinite(out).all()
    assert np.linalg.norm(ref) > 0
    e_acc = O.rel_l2(acc, ref)
    e_out = O.rel_l2(out, O.bf16_round(ref))
    assert e_acc <= TOL, f"{name}: fp32 accumulator rel-L2 {e_acc:.3e}"
    assert e_out <= TOL, f"{name}: bf16 output rel-L2 vs bf16(oracle) {e_out:.3e}"
