"""The CTA-pair forward kernel (head_dim 128, two query tiles per cluster of two
CTAs, M = 256 tensor-core products) against the fp64 oracle and against the
one-CTA-per-tile kernel, through the public API.

The pair kernel is chosen once per process (TDA_B200_FWD_PAIR=1), so each
schedule runs the same cases in a child process.  Cases cover the pair's own
edges: an odd number of query tiles (the last pair's odd CTA lies past the
sequence), ragged S, a single tile, S of 64, beta = 0 (dense P) and beta < 0
(every key tile, masked entries included), every power branch, normalize off,
fp16 inputs, (B, S, H, D) views read in place, and a per-head lambda on the
device.

Checks:
  * fp32 accumulator output vs the oracle <= 1e-3, bf16 output vs the
    bf16-rounded oracle <= 1e-3 (as every bf16 parity test here);
  * pair vs one-tile kernel: bit-identical.  Both run the same products per
    query row in the same order; a 16-key slab the pair skips holds P = 0 in
    both of its tiles, so skipping it adds exactly nothing.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import tda_oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
TOL = 1e-3

# name: (op, (B, H, S), beta, lam, p, normalize, dtype, layout, lam_kind)
CASES = {
    "diff_ragged_even": ("diff", (2, 3, 1000), 1.0, 0.5, 2.0, True, "bf16", "bhsd", "scalar"),
    "diff_odd_tiles": ("diff", (1, 2, 1300), 1.0, 0.5, 2.0, True, "bf16", "bhsd", "scalar"),
    "rect_even": ("rect", (2, 2, 1536), 1.0, 0.0, 2.0, True, "bf16", "bhsd", "scalar"),
    "rect_odd_tiles": ("rect", (1, 3, 520), 1.0, 0.0, 2.0, True, "bf16", "bhsd", "scalar"),
    "diff_one_tile": ("diff", (1, 2, 128), 1.0, 0.5, 2.0, True, "bf16", "bhsd", "scalar"),
    "rect_s64": ("rect", (1, 2, 64), 0.5, 0.0, 2.0, True, "bf16", "bhsd", "scalar"),
    "diff_dense_beta0": ("diff", (1, 2, 1024), 0.0, 0.5, 2.0, True, "bf16", "bhsd", "scalar"),
    "diff_beta_neg": ("diff", (1, 2, 800), -0.5, 0.5, 2.0, True, "bf16", "bhsd", "scalar"),
    "rect_beta_neg_p3": ("rect", (1, 2, 640), -0.5, 0.0, 3.0, True, "bf16", "bhsd", "scalar"),
    "diff_p1": ("diff", (1, 2, 512), 1.0, 0.3, 1.0, True, "bf16", "bhsd", "scalar"),
    "diff_p3": ("diff", (1, 2, 512), 1.0, 0.7, 3.0, True, "bf16", "bhsd", "scalar"),
    "diff_p1_5": ("diff", (1, 2, 512), 1.0, 0.6, 1.5, True, "bf16", "bhsd", "scalar"),
    "rect_p1_5": ("rect", (1, 2, 384), 0.5, 0.0, 1.5, True, "bf16", "bhsd", "scalar"),
    "diff_no_norm": ("diff", (1, 2, 384), 0.5, 0.5, 2.0, False, "bf16", "bhsd", "scalar"),
    "rect_no_norm_beta_neg": ("rect", (1, 2, 300), -0.5, 0.0, 2.0, False, "bf16", "bhsd", "scalar"),
    "diff_fp16": ("diff", (1, 2, 768), 1.0, 0.5, 2.0, True, "f16", "bhsd", "scalar"),
    "rect_fp16_odd": ("rect", (1, 2, 650), 1.0, 0.0, 2.0, True, "f16", "bhsd", "scalar"),
    "diff_bshd_views": ("diff", (2, 3, 700), 1.0, 0.5, 2.0, True, "bf16", "bshd", "scalar"),
    "diff_lambda_per_head": ("diff", (2, 3, 600), 1.0, 0.0, 2.0, True, "bf16", "bhsd", "per_head"),
}
D = 128

CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
import tda_b200
from test_gpu_pair import CASES, make_inputs, lam_of
res = {}
for name in sys.argv[2].split(","):
    op, (B, H, S), beta, lam, p, norm, dt, layout, lam_kind = CASES[name]
    xs = [x.cuda() for x in make_inputs(name)]
    if layout == "bshd":
        xs = [x.transpose(1, 2).contiguous().transpose(1, 2) for x in xs]
    lam_t = lam_of(name).cuda() if lam_kind == "per_head" else torch.tensor(lam)
    if op == "diff":
        acc = tda_b200.diff_forward(*xs, beta, lam_t.cuda() if lam_kind == "per_head" else lam, p, norm,
                                    out_dtype=torch.float32)
        out = tda_b200.differential_threshold_rela_triton(*xs, torch.tensor(beta), lam_t, p, norm)
    else:
        acc = tda_b200.rect_forward(xs[0], xs[1], xs[2], beta, p, norm, out_dtype=torch.float32)
        out = tda_b200.threshold_rela_triton(xs[0], xs[1], xs[2], torch.tensor(beta), p, norm)
    tda_b200.check_status()
    res[name + "/acc"] = acc.float().cpu().numpy()
    res[name + "/out"] = out.float().cpu().numpy()
np.savez(sys.argv[3], **res)
"""


def make_inputs(name):
    """Seeded N(0,1) inputs of a case on the CPU, (B, H, S, D), in the case's dtype."""
    import torch
    op, (B, H, S), *_rest = CASES[name]
    dt = {"bf16": torch.bfloat16, "f16": torch.float16}[CASES[name][6]]
    g = torch.Generator(device="cpu").manual_seed(1_000_003 + sum(map(ord, name)))
    n = 5 if op == "diff" else 3
    return [torch.randn((B, H, S, D), generator=g).to(dt) for _ in range(n)]


def lam_of(name):
    import torch
    H = CASES[name][1][1]
    return torch.linspace(0.1, 0.9, H).view(1, H, 1, 1)


def _oracle(name):
    op, (B, H, S), beta, lam, p, norm, dt, layout, lam_kind = CASES[name]
    xn = [x.float().numpy() for x in make_inputs(name)]
    if op == "rect":
        return O.rect_fwd(xn[0], xn[1], xn[2], beta, p, norm)
    if lam_kind != "per_head":
        return O.diff_fwd(*xn, beta, lam, p, norm)
    lams = lam_of(name).view(-1).numpy()
    out = np.zeros(xn[0].shape)
    for h in range(H):
        out[:, h:h + 1] = O.diff_fwd(*[x[:, h:h + 1] for x in xn], beta, float(lams[h]), p, norm)
    return out


def _run(tmp_path_factory, pair):
    path = str(tmp_path_factory.mktemp("pair") / f"pair{pair}.npz")
    env = dict(os.environ, TDA_B200_FWD_PAIR=pair, TDA_B200_FWD_PERSISTENT="0")
    subprocess.run([sys.executable, "-c", CHILD, ROOT, ",".join(CASES), path], env=env, check=True, timeout=900)
    return np.load(path)


@pytest.fixture(scope="module")
def results(tmp_path_factory):
    return _run(tmp_path_factory, "1"), _run(tmp_path_factory, "0")


@pytest.mark.parametrize("name", list(CASES))
def test_pair_kernel_matches_oracle_and_one_tile_kernel(results, name):
    pair, tile = results
    ref = _oracle(name)
    acc, out = pair[name + "/acc"], pair[name + "/out"]
    assert np.isfinite(acc).all() and np.isfinite(out).all()
    e_acc = O.rel_l2(acc, ref)
    round_ = O.bf16_round if CASES[name][6] == "bf16" else (lambda x: x.astype(np.float16).astype(np.float64))
    e_out = O.rel_l2(out, round_(ref))
    assert e_acc <= TOL, f"{name}: fp32 accumulator rel-L2 {e_acc:.3e}"
    assert e_out <= TOL, f"{name}: output rel-L2 vs rounded oracle {e_out:.3e}"
    assert np.array_equal(acc, tile[name + "/acc"]), f"{name}: pair and one-tile accumulators differ"
    assert np.array_equal(out, tile[name + "/out"]), f"{name}: pair and one-tile outputs differ"
