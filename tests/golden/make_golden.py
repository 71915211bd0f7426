"""Generate golden vectors by running the reference TDA implementation on CPU.

The reference (snap-research/TDA, ``triton_threshold_attention.py``) is a Triton
program; with ``TRITON_INTERPRET=1`` its kernels run on CPU tensors in numpy
float32.  This script imports it from a reference checkout, feeds it seeded
inputs and writes ``golden_cases.npz`` next to itself: the inputs, the
parameters and the reference's outputs for every case in ``CASES``.

It needs the reference checkout, so it runs only where that exists:

    python tests/golden/make_golden.py --reference <path to the TDA checkout>

The committed ``golden_cases.npz`` is what the tests read; nothing at test time
touches the reference.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# name, op, (B,H,S,D), dtype, params
#   op "rect": threshold_rela_triton(q,k,v,beta,p) on (optionally) F.normalize'd q,k
#   op "diff": differential_threshold_rela_triton(q1,q2,k1,k2,v,beta,lam,p,normalize)
CASES = [
    ("rect_basic", "rect", (1, 2, 64, 64), "f32", dict(beta=1.0, p=2.0, normalize=False, std=1.0)),
    ("rect_norm", "rect", (1, 2, 64, 64), "f32", dict(beta=1.0, p=2.0, normalize=True, std=1.0)),
    ("rect_cfg1", "rect", (1, 8, 128, 64), "f32", dict(beta=1.0, p=2.0, normalize=True, std=1.0)),
    ("rect_ragged_s100", "rect", (1, 2, 100, 64), "f32", dict(beta=1.0, p=2.0, normalize=False, std=1.0)),
    ("rect_s1", "rect", (1, 1, 1, 64), "f32", dict(beta=1.0, p=2.0, normalize=False, std=1.0)),
    ("rect_s65", "rect", (2, 1, 65, 32), "f32", dict(beta=0.5, p=2.0, normalize=True, std=1.0)),
    ("rect_p1", "rect", (1, 2, 64, 64), "f32", dict(beta=0.5, p=1.0, normalize=False, std=1.0)),
    ("rect_p3", "rect", (1, 2, 64, 64), "f32", dict(beta=1.0, p=3.0, normalize=False, std=1.0)),
    ("rect_p1_5", "rect", (1, 2, 64, 64), "f32", dict(beta=2.0, p=1.5, normalize=True, std=2.0)),
    ("rect_beta0", "rect", (1, 2, 64, 64), "f32", dict(beta=0.0, p=2.0, normalize=True, std=1.0)),
    ("rect_beta_neg", "rect", (1, 2, 64, 64), "f32", dict(beta=-0.5, p=2.0, normalize=False, std=1.0)),
    ("rect_beta_neg_norm", "rect", (1, 2, 96, 64), "f32", dict(beta=-1.0, p=2.0, normalize=True, std=1.0)),
    ("rect_d128", "rect", (1, 2, 64, 128), "f32", dict(beta=1.0, p=2.0, normalize=True, std=1.0)),
    ("rect_d16", "rect", (1, 2, 48, 16), "f32", dict(beta=1.0, p=2.0, normalize=False, std=1.0)),
    ("rect_std2_p3", "rect", (1, 1, 128, 64), "f32", dict(beta=2.0, p=3.0, normalize=False, std=2.0)),
    ("diff_basic", "diff", (1, 2, 64, 64), "f32", dict(beta=1.0, lam=0.5, p=2.0, normalize=True, std=1.0)),
    ("diff_nonorm", "diff", (1, 2, 64, 64), "f32", dict(beta=0.5, lam=0.3, p=2.0, normalize=False, std=1.0)),
    ("diff_lam_clamp_hi", "diff", (1, 1, 64, 64), "f32", dict(beta=1.0, lam=1.5, p=2.0, normalize=True, std=1.0)),
    ("diff_lam_clamp_lo", "diff", (1, 1, 64, 64), "f32", dict(beta=1.0, lam=-0.25, p=2.0, normalize=True, std=1.0)),
    ("diff_ragged_p3", "diff", (1, 2, 77, 64), "f32", dict(beta=0.5, lam=0.8, p=3.0, normalize=True, std=1.0)),
    ("diff_beta_neg", "diff", (1, 1, 80, 64), "f32", dict(beta=-0.7, lam=0.5, p=2.0, normalize=True, std=1.0)),
    ("diff_d128", "diff", (1, 1, 128, 128), "f32", dict(beta=1.5, lam=0.8, p=2.0, normalize=True, std=1.0)),
    # bf16 cases record the reference's own bf16 behaviour (upcast to fp32 inside
    # the op, downcast of the result; in the differential form F.normalize and
    # the combine also run in bf16).
    ("rect_bf16", "rect", (1, 2, 128, 64), "bf16", dict(beta=1.0, p=2.0, normalize=False, std=1.0)),
    ("rect_bf16_d128", "rect", (1, 1, 130, 128), "bf16", dict(beta=0.5, p=2.0, normalize=False, std=1.0)),
    ("diff_bf16", "diff", (1, 2, 128, 64), "bf16", dict(beta=1.0, lam=0.5, p=2.0, normalize=True, std=1.0)),
]


def gen_inputs(seed: int, n: int, shape, dtype: str, std: float):
    """n tensors of i.i.d. N(0, std^2) entries from a seeded PCG64 generator.
    bf16 cases are rounded to bf16 (returned widened to fp32)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    xs = [(rng.standard_normal(shape, dtype=np.float32) * np.float32(std)) for _ in range(n)]
    if dtype == "bf16":
        import torch
        xs = [torch.from_numpy(x).bfloat16().float().numpy() for x in xs]
    return xs


def run_case(T, torch, name, op, shape, dtype, prm, seed):
    F = torch.nn.functional
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    beta = torch.tensor(prm["beta"])
    if op == "rect":
        q, k, v = gen_inputs(seed, 3, shape, dtype, prm["std"])
        tq, tk, tv = (torch.from_numpy(x).to(tdt) for x in (q, k, v))
        if prm["normalize"]:
            tq, tk = F.normalize(tq, p=2, dim=-1), F.normalize(tk, p=2, dim=-1)
        out = T.threshold_rela_triton(tq, tk, tv, beta, prm["p"])
        arrays = dict(q=q, k=k, v=v)
    else:
        q1, q2, k1, k2, v = gen_inputs(seed, 5, shape, dtype, prm["std"])
        t = [torch.from_numpy(x).to(tdt) for x in (q1, q2, k1, k2, v)]
        out = T.differential_threshold_rela_triton(
            t[0], t[1], t[2], t[3], t[4], beta, torch.tensor(prm["lam"]), prm["p"], prm["normalize"])
        arrays = dict(q1=q1, q2=q2, k1=k1, k2=k2, v=v)
    assert out.dtype == tdt, (name, out.dtype)
    arrays["out"] = out.float().numpy()
    return arrays


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory holding triton_threshold_attention.py")
    ap.add_argument("--out", default=os.path.join(HERE, "golden_cases.npz"))
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    import triton_threshold_attention as T  # the reference, run by the Triton interpreter

    blob = {}
    meta = []
    for i, (name, op, shape, dtype, prm) in enumerate(CASES):
        seed = 1000 + i
        arrays = run_case(T, torch, name, op, shape, dtype, prm, seed)
        for key, val in arrays.items():
            blob[f"{name}/{key}"] = np.ascontiguousarray(val, dtype=np.float32)
        meta.append(dict(name=name, op=op, shape=list(shape), dtype=dtype, seed=seed, **prm))
        print(f"{name}: done", flush=True)
    blob["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **blob)
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
