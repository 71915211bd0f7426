"""Pin the CPU oracle against outputs of the reference implementation itself.

The golden vectors were produced by running the reference
(triton_threshold_attention.py) on CPU under TRITON_INTERPRET=1
(tests/golden/make_golden.py).  The reference computes in fp32 there, so the
fp64 oracle must agree to fp32 rounding.
"""
import numpy as np
import pytest

from golden_io import load_cases
from oracle import tda_oracle as O

CASES = load_cases()
F32 = [c for c in CASES if c[0]["dtype"] == "f32"]
BF16 = [c for c in CASES if c[0]["dtype"] == "bf16"]


def _oracle(m, a, dtype=np.float64):
    if m["op"] == "rect":
        return O.rect_fwd(a["q"], a["k"], a["v"], m["beta"], m["p"], m["normalize"], dtype=dtype)
    return O.diff_fwd(a["q1"], a["q2"], a["k1"], a["k2"], a["v"], m["beta"], m["lam"], m["p"], m["normalize"],
                      dtype=dtype)


@pytest.mark.parametrize("case", F32, ids=[c[0]["name"] for c in F32])
def test_oracle_matches_reference_fp32(case):
    m, a = case
    o = _oracle(m, a)
    assert O.rel_l2(a["out"], o) <= 1e-5


@pytest.mark.parametrize("case", F32, ids=[c[0]["name"] for c in F32])
def test_oracle_fp32_mode_matches_reference(case):
    # the fp32 formula (what the CPU baseline times) tracks the reference too
    m, a = case
    o = _oracle(m, a, dtype=np.float32)
    assert O.rel_l2(a["out"], o) <= 1e-5


def _bf16_reference_emulation(m, a):
    """The reference's own bf16 pipeline, step by step: F.normalize and the
    combine run in bf16 (:505-509, :516-517); each rect call upcasts to fp32,
    computes, and rounds its output to bf16 (:356-360, :392-393)."""
    r = O.bf16_round

    def norm_bf16(x):
        x = np.asarray(x, np.float32)
        n = r(np.sqrt(np.sum(x.astype(np.float32) ** 2, axis=-1, keepdims=True, dtype=np.float32)))
        return r(x / np.maximum(n, np.float32(1e-12)))

    if m["op"] == "rect":
        return r(O.rect_fwd(a["q"], a["k"], a["v"], m["beta"], m["p"], False, dtype=np.float32))
    q1, q2, k1, k2 = a["q1"], a["q2"], a["k1"], a["k2"]
    if m["normalize"]:
        q1, q2, k1, k2 = (norm_bf16(x) for x in (q1, q2, k1, k2))
    o1 = r(O.rect_fwd(q1, k1, a["v"], m["beta"], m["p"], False, dtype=np.float32))
    o2 = r(O.rect_fwd(q2, k2, a["v"], m["beta"], m["p"], False, dtype=np.float32))
    lam = np.float32(min(max(m["lam"], 0.0), 1.0))
    return r(o1 - r(lam * o2))


@pytest.mark.parametrize("case", BF16, ids=[c[0]["name"] for c in BF16])
def test_reference_bf16_semantics_understood(case):
    """The oracle's model of the reference's bf16 rounding steps reproduces its
    bf16 outputs (up to single-ulp flips), while the exact math differs from
    them by the reference's own bf16 error."""
    m, a = case
    emu = _bf16_reference_emulation(m, a)
    assert O.rel_l2(emu, a["out"]) <= 2e-3
    exact = _oracle(m, a)
    if m["op"] == "diff" and m["normalize"]:
        # bf16 F.normalize before the threshold costs the reference ~1e-2
        assert O.rel_l2(a["out"], exact) > 1e-3


def test_tau_formula():
    tau = O.tau_vector(8, 64, 1.0)
    assert tau[0] == 0.0
    np.testing.assert_allclose(tau[7], np.sqrt(2 * np.log(8.0) / 64), rtol=1e-6)


def test_mask_to_zero_semantics_negative_beta():
    # beta < 0: masked (future) keys contribute relu(0 - tau)^p v_j (:79-80)
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 1, 5, 16)) for _ in range(3))
    out = O.rect_fwd(q, k, v, -1.0, 2.0, False)
    tau = O.tau_vector(5, 16, -1.0).astype(np.float64)
    s = q[0, 0] @ k[0, 0].T
    s = np.where(np.tril(np.ones((5, 5), bool)), s, 0.0)
    P = np.maximum(s - tau[:, None], 0.0) ** 2
    np.testing.assert_allclose(out[0, 0], P @ v[0, 0], rtol=1e-12)
    # row 1 (tau_1 < 0) sees its future keys through the mask-to-zero; row 0 has tau = 0
    assert np.all(P[1, 2:] > 0) and np.all(P[0] == np.maximum(np.where(np.arange(5) == 0, s[0, 0], 0.0), 0) ** 2)
