"""Generate backward golden vectors by running the reference TDA implementation on CPU.

Same arrangement as ``make_golden.py``: the reference (snap-research/TDA,
``triton_threshold_attention.py``) runs under ``TRITON_INTERPRET=1``; inputs are
seeded, torch autograd drives the reference's own backward
(``ThresholdRelaFunction.backward`` and its two Triton kernels, plus torch's
gradients for F.normalize, clamp and the combine in the differential form),
and the gradients are written to ``golden_bwd.npz`` next to this script:

    python tests/golden/make_golden_bwd.py --reference <path to the TDA checkout>

The committed ``golden_bwd.npz`` is what the tests read; nothing at test time
touches the reference.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# name, op, (B,H,S,D), params -- all fp32
CASES = [
    ("rect_basic", "rect", (1, 2, 64, 64), dict(beta=1.0, p=2.0, normalize=False, std=1.0)),
    ("rect_norm", "rect", (1, 2, 64, 64), dict(beta=1.0, p=2.0, normalize=True, std=1.0)),
    ("rect_p1", "rect", (1, 2, 64, 64), dict(beta=0.5, p=1.0, normalize=False, std=1.0)),
    ("rect_p3", "rect", (1, 1, 64, 64), dict(beta=1.0, p=3.0, normalize=False, std=1.0)),
    ("rect_p1_5_norm", "rect", (1, 2, 64, 64), dict(beta=2.0, p=1.5, normalize=True, std=2.0)),
    ("rect_beta0_norm", "rect", (1, 1, 64, 64), dict(beta=0.0, p=2.0, normalize=True, std=1.0)),
    ("rect_beta_neg", "rect", (1, 2, 64, 64), dict(beta=-0.5, p=2.0, normalize=False, std=1.0)),
    ("rect_beta_neg_norm", "rect", (1, 1, 96, 64), dict(beta=-1.0, p=2.0, normalize=True, std=1.0)),
    ("rect_ragged_s100", "rect", (1, 1, 100, 32), dict(beta=1.0, p=2.0, normalize=False, std=1.0)),
    ("rect_d128_norm", "rect", (1, 1, 64, 128), dict(beta=1.0, p=2.0, normalize=True, std=1.0)),
    ("diff_basic", "diff", (1, 2, 64, 64), dict(beta=1.0, lam=0.5, p=2.0, normalize=True, std=1.0)),
    ("diff_nonorm", "diff", (1, 1, 64, 64), dict(beta=0.5, lam=0.3, p=2.0, normalize=False, std=1.0)),
    ("diff_lam_clamp_hi", "diff", (1, 1, 64, 64), dict(beta=1.0, lam=1.5, p=2.0, normalize=True, std=1.0)),
    ("diff_lam_clamp_lo", "diff", (1, 1, 64, 64), dict(beta=1.0, lam=-0.25, p=2.0, normalize=True, std=1.0)),
    ("diff_ragged_p3", "diff", (1, 1, 77, 64), dict(beta=0.5, lam=0.8, p=3.0, normalize=True, std=1.0)),
    ("diff_beta_neg", "diff", (1, 1, 80, 64), dict(beta=-0.7, lam=0.5, p=2.0, normalize=True, std=1.0)),
]


def gen_inputs(seed: int, n: int, shape, std: float):
    """n tensors of i.i.d. N(0, std^2) entries from a seeded PCG64 generator,
    then the upstream gradient dout ~ N(0, 1)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    xs = [(rng.standard_normal(shape, dtype=np.float32) * np.float32(std)) for _ in range(n)]
    dout = rng.standard_normal(shape, dtype=np.float32)
    return xs, dout


def run_case(T, torch, name, op, shape, prm, seed):
    F = torch.nn.functional
    beta = torch.tensor(prm["beta"])
    if op == "rect":
        (q, k, v), dout = gen_inputs(seed, 3, shape, prm["std"])
        t = [torch.from_numpy(x).clone().requires_grad_(True) for x in (q, k, v)]
        tq, tk = t[0], t[1]
        if prm["normalize"]:
            tq, tk = F.normalize(tq, p=2, dim=-1), F.normalize(tk, p=2, dim=-1)
        out = T.threshold_rela_triton(tq, tk, t[2], beta, prm["p"])
        out.backward(torch.from_numpy(dout))
        arrays = dict(q=q, k=k, v=v, dout=dout, out=out.detach().numpy(),
                      dq=t[0].grad.numpy(), dk=t[1].grad.numpy(), dv=t[2].grad.numpy())
    else:
        (q1, q2, k1, k2, v), dout = gen_inputs(seed, 5, shape, prm["std"])
        t = [torch.from_numpy(x).clone().requires_grad_(True) for x in (q1, q2, k1, k2, v)]
        lam = torch.tensor(prm["lam"], requires_grad=True)
        out = T.differential_threshold_rela_triton(t[0], t[1], t[2], t[3], t[4], beta, lam, prm["p"],
                                                   prm["normalize"])
        out.backward(torch.from_numpy(dout))
        arrays = dict(q1=q1, q2=q2, k1=k1, k2=k2, v=v, dout=dout, out=out.detach().numpy(),
                      dq1=t[0].grad.numpy(), dq2=t[1].grad.numpy(), dk1=t[2].grad.numpy(),
                      dk2=t[3].grad.numpy(), dv=t[4].grad.numpy(),
                      dlam=np.asarray([lam.grad.item()], dtype=np.float32))
    return arrays


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory holding triton_threshold_attention.py")
    ap.add_argument("--out", default=os.path.join(HERE, "golden_bwd.npz"))
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    import triton_threshold_attention as T  # the reference, run by the Triton interpreter

    blob = {}
    meta = []
    for i, (name, op, shape, prm) in enumerate(CASES):
        seed = 5000 + i
        arrays = run_case(T, torch, name, op, shape, prm, seed)
        for key, val in arrays.items():
            blob[f"{name}/{key}"] = np.ascontiguousarray(val, dtype=np.float32)
        meta.append(dict(name=name, op=op, shape=list(shape), dtype="f32", seed=seed, **prm))
        print(f"{name}: done", flush=True)
    blob["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **blob)
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
