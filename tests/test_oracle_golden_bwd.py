"""The backward oracle against the reference's own gradients (CPU only).

tests/golden/golden_bwd.npz holds gradients that torch autograd produced through
the reference op run under the Triton interpreter (make_golden_bwd.py): dq, dk,
dv of threshold_rela_triton (on F.normalize'd q, k when normalize), and dq1, dq2,
dk1, dk2, dv, d lambda of differential_threshold_rela_triton.  The reference ran
in fp32, the oracle runs in fp64, so they agree to fp32 rounding.  The beta < 0
cases pin the reference's handling of masked entries in dQ / dK."""
import numpy as np
import pytest

from golden_io import load_bwd_cases
from oracle import tda_oracle as O

CASES = load_bwd_cases()
TOL = 2e-5


@pytest.mark.parametrize("meta,arrays", CASES, ids=[m["name"] for m, _ in CASES])
def test_oracle_backward_matches_reference(meta, arrays):
    if meta["op"] == "rect":
        got = O.rect_bwd(arrays["q"], arrays["k"], arrays["v"], arrays["dout"], meta["beta"], meta["p"],
                         meta["normalize"])
        names = ("dq", "dk", "dv")
    else:
        got = O.diff_bwd(arrays["q1"], arrays["q2"], arrays["k1"], arrays["k2"], arrays["v"], arrays["dout"],
                         meta["beta"], meta["lam"], meta["p"], meta["normalize"])
        names = ("dq1", "dq2", "dk1", "dk2", "dv", "dlam")
    for name, g in zip(names, got):
        ref = arrays[name]
        if name == "dlam":
            assert abs(g - float(ref[0])) <= TOL * max(1.0, abs(float(ref[0]))), (g, ref)
        else:
            err = O.rel_l2(g, ref)
            assert err <= TOL, (name, err)


def test_masked_entry_quirk_is_visible_for_negative_beta():
    """With beta < 0 the reference's dQ includes keys after the query row; the
    exact gradient of the forward would not.  The golden case shows the
    difference is material, so the oracle must keep it."""
    meta, arrays = next(c for c in CASES if c[0]["name"] == "rect_beta_neg")
    dq, _, _ = O.rect_bwd(arrays["q"], arrays["k"], arrays["v"], arrays["dout"], meta["beta"], meta["p"], False)
    # exact gradient: drop the masked entries' contribution
    q, k, v, g = (arrays[n].astype(np.float64) for n in ("q", "k", "v", "dout"))
    S, D = q.shape[2], q.shape[3]
    tau = O.tau_vector(S, D, meta["beta"]).astype(np.float64)
    mask = np.tril(np.ones((S, S), dtype=bool))
    s = np.where(mask, q @ np.swapaxes(k, -1, -2), 0.0)
    z = s - tau[:, None]
    dA = (g @ np.swapaxes(v, -1, -2)) * O.relu_power_grad(z, 2.0) * mask
    exact = dA @ k
    assert O.rel_l2(dq, arrays["dq"]) <= TOL
    assert O.rel_l2(exact, arrays["dq"]) > 1e-2
