"""Backward pass of the CUDA path against the backward oracle, which is pinned
to the reference's own gradients (tests/test_oracle_golden_bwd.py).

Paths and tolerances (rel-L2):
  * fp32 inputs (and head_dim 16 / 32 / 256): exact fp32 on CUDA cores,
    fp32 gradients vs the fp64 oracle                                <= 1e-5
  * bf16 inputs, head_dim 64 / 128: tcgen05 tensor cores, bf16 operands with
    P and dA as bf16 hi + lo, fp32 accumulation; fp32 gradients
    (``rect_backward``) vs the fp64 oracle on the bf16 values         <= 2e-5
  * through autograd, bf16 gradients vs the bf16-rounded oracle      <= 1e-3
"""
import numpy as np
import pytest
import torch

import tda_b200
from golden_io import load_bwd_cases
from oracle import tda_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL_F32 = 1e-5
TOL_TC = 2e-5
TOL_BF16 = 1e-3


def _t(x, dtype=torch.float32, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(DEV).to(dtype)
    return t.requires_grad_(grad)


def _np(t):
    return t.detach().float().cpu().numpy()


def _gen(seed, n, shape, std=1.0, dtype=torch.float32):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return [(torch.randn(shape, generator=g) * std).to(dtype) for _ in range(n)]


BWD_CASES = load_bwd_cases()


@pytest.mark.parametrize("case", BWD_CASES, ids=[c[0]["name"] for c in BWD_CASES])
def test_golden_backward_through_autograd(case):
    """The reference's gradients (autograd through the reference op) vs ours
    through the public API's autograd, fp32."""
    m, a = case
    beta = torch.tensor(m["beta"])
    if m["op"] == "rect":
        q, k, v = (_t(a[n], grad=True) for n in ("q", "k", "v"))
        out = tda_b200.threshold_rela_triton(q, k, v, beta, m["p"], m["normalize"])
        out.backward(_t(a["dout"]))
        ref = O.rect_bwd(a["q"], a["k"], a["v"], a["dout"], m["beta"], m["p"], m["normalize"])
        got = (q.grad, k.grad, v.grad)
        names = ("dq", "dk", "dv")
    else:
        xs = [_t(a[n], grad=True) for n in ("q1", "q2", "k1", "k2", "v")]
        lam = torch.tensor(m["lam"], device=DEV, requires_grad=True)
        out = tda_b200.differential_threshold_rela_triton(*xs, beta, lam, m["p"], m["normalize"])
        out.backward(_t(a["dout"]))
        ref = O.diff_bwd(a["q1"], a["q2"], a["k1"], a["k2"], a["v"], a["dout"], m["beta"], m["lam"], m["p"],
                         m["normalize"])
        got = tuple(x.grad for x in xs) + (lam.grad,)
        names = ("dq1", "dq2", "dk1", "dk2", "dv", "dlam")
    tda_b200.check_status()
    for name, g_ours, g_oracle in zip(names, got, ref):
        if name == "dlam":
            assert abs(float(g_ours) - g_oracle) <= 1e-4 * max(1.0, abs(g_oracle)), (float(g_ours), g_oracle)
            assert abs(float(g_ours) - float(a["dlam"][0])) <= 1e-4 * max(1.0, abs(g_oracle))
            continue
        assert O.rel_l2(_np(g_ours), g_oracle) <= TOL_F32, (name, O.rel_l2(_np(g_ours), g_oracle))
        # and the reference's own fp32 gradients
        assert O.rel_l2(_np(g_ours), a[name]) <= 5e-5, (name, O.rel_l2(_np(g_ours), a[name]))


@pytest.mark.parametrize("D", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("beta,p,norm", [(1.0, 2.0, True), (0.5, 3.0, False), (-0.5, 2.0, True),
                                         (1.5, 1.0, True), (2.0, 1.5, False)])
def test_rect_backward_fp32_tiles(D, beta, p, norm):
    """Several 64-row tiles (32-row at head_dim 256), a ragged last tile, both
    tile loops, every head dim."""
    q, k, v, g = _gen(100 + D, 4, (1, 2, 200, D))
    dq, dk, dv = tda_b200.rect_backward(*(x.to(DEV) for x in (q, k, v, g)), beta, p, norm)
    ref = O.rect_bwd(q.numpy(), k.numpy(), v.numpy(), g.numpy(), beta, p, norm)
    for got, r, name in zip((dq, dk, dv), ref, ("dq", "dk", "dv")):
        assert O.rel_l2(_np(got), r) <= TOL_F32, (name, O.rel_l2(_np(got), r))


@pytest.mark.parametrize("D", [64, 128])
def test_rect_backward_bf16_inputs(D):
    """bf16 q, k, v, dout: exact fp32 gradients from the bf16 values, and the
    bf16 gradients autograd hands back."""
    q, k, v, g = _gen(200 + D, 4, (2, 2, 256, D), dtype=torch.bfloat16)
    dq, dk, dv = tda_b200.rect_backward(*(x.to(DEV) for x in (q, k, v, g)), 1.0, 2.0, True)
    ref = O.rect_bwd(*(x.float().numpy() for x in (q, k, v, g)), 1.0, 2.0, True)
    for got, r in zip((dq, dk, dv), ref):
        assert O.rel_l2(_np(got), r) <= TOL_TC
    qg, kg, vg = (x.to(DEV).requires_grad_(True) for x in (q, k, v))
    out = tda_b200.threshold_rela_triton(qg, kg, vg, 1.0, 2.0, True)
    out.backward(g.to(DEV))
    for got, r in zip((qg.grad, kg.grad, vg.grad), ref):
        assert got.dtype == torch.bfloat16
        assert O.rel_l2(_np(got), O.bf16_round(r)) <= TOL_BF16


def test_head_dim_256_backward_through_autograd():
    """head_dim 256 (the reference's kernels take any power-of-two BLOCK_D,
    :368, :436-460): bf16 inputs through the differential form's autograd on
    the CUDA-core kernels with 32-row tiles, exact fp32 gradients of the bf16
    values, handed back in bf16."""
    xs = _gen(700, 6, (1, 2, 150, 256), dtype=torch.bfloat16)
    ins = [x.to(DEV).requires_grad_(True) for x in xs[:5]]
    lam = torch.tensor(0.4, device=DEV, requires_grad=True)
    out = tda_b200.differential_threshold_rela_triton(*ins, 0.5, lam, 2.0, True)
    out.backward(xs[5].to(DEV))
    ref = O.diff_bwd(*[x.float().numpy() for x in xs[:5]], xs[5].float().numpy(), 0.5, 0.4, 2.0, True)
    for got, r in zip(ins, ref[:5]):
        assert got.grad.dtype == torch.bfloat16
        assert O.rel_l2(_np(got.grad), O.bf16_round(r)) <= TOL_BF16
    assert abs(float(lam.grad) - ref[5]) <= 1e-3 * max(1.0, abs(ref[5]))
    tda_b200.check_status()


def test_diff_backward_per_head_lambda():
    """A per-head lambda (broadcast (1, H, 1, 1)), one head clamped: d lambda
    per head, and the second branch scaled per head."""
    xs = _gen(300, 6, (1, 3, 130, 64))
    lam0 = torch.tensor([0.25, 0.75, 1.4]).reshape(1, 3, 1, 1)
    ins = [x.to(DEV).requires_grad_(True) for x in xs[:5]]
    lam = lam0.to(DEV).requires_grad_(True)
    out = tda_b200.differential_threshold_rela_triton(*ins, 1.0, lam, 2.0, True)
    out.backward(xs[5].to(DEV))
    for h in range(3):
        sl = [x[:, h:h + 1].numpy() for x in xs]
        ref = O.diff_bwd(*sl[:5], sl[5], 1.0, float(lam0[0, h]), 2.0, True)
        for t, r in zip(ins, ref[:5]):
            assert O.rel_l2(_np(t.grad[:, h:h + 1]), r) <= TOL_F32
        assert abs(float(lam.grad[0, h]) - ref[5]) <= 1e-4 * max(1.0, abs(ref[5]))


def test_backward_accumulates_dv():
    q, k, v, g = (x.to(DEV) for x in _gen(400, 4, (1, 1, 96, 32)))
    _, _, dv1 = tda_b200.rect_backward(q, k, v, g, 1.0, 2.0, False)
    dv = dv1.clone()
    tda_b200.rect_backward(q, k, v, g, 1.0, 2.0, False, dout_scale=-0.5, dv=dv)
    assert O.rel_l2(_np(dv), 0.5 * _np(dv1)) <= 1e-6


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("shape_s,beta,p,norm", [(256, 1.0, 2.0, True), (200, 0.5, 3.0, False),
                                                 (300, -0.5, 2.0, True), (256, 0.0, 1.0, True),
                                                 (130, 1.5, 1.5, True), (129, -1.0, 2.0, False)])
def test_tensor_core_backward_sweep(D, shape_s, beta, p, norm):
    """The tcgen05 backward (bf16) over thresholds, powers, normalize, ragged
    lengths and negative beta (masked entries kept in dQ / dK)."""
    q, k, v, g = _gen(500 + shape_s + D, 4, (1, 2, shape_s, D), dtype=torch.bfloat16)
    dq, dk, dv = tda_b200.rect_backward(*(x.to(DEV) for x in (q, k, v, g)), beta, p, norm)
    tda_b200.check_status()
    ref = O.rect_bwd(*(x.float().numpy() for x in (q, k, v, g)), beta, p, norm)
    for got, r, name in zip((dq, dk, dv), ref, ("dq", "dk", "dv")):
        assert O.rel_l2(_np(got), r) <= TOL_TC, (name, O.rel_l2(_np(got), r))


def test_tensor_core_diff_backward_matches_oracle():
    """Both branches of the differential form on the tensor cores (bf16, D 128)."""
    xs = _gen(600, 6, (1, 2, 256, 128), dtype=torch.bfloat16)
    ins = [x.to(DEV).requires_grad_(True) for x in xs[:5]]
    lam = torch.tensor(0.6, device=DEV, requires_grad=True)
    out = tda_b200.differential_threshold_rela_triton(*ins, 1.0, lam, 2.0, True)
    out.backward(xs[5].to(DEV))
    ref = O.diff_bwd(*(x.float().numpy() for x in xs[:5]), xs[5].float().numpy(), 1.0, 0.6, 2.0, True)
    for t, r in zip(ins, ref[:5]):
        assert O.rel_l2(_np(t.grad), O.bf16_round(r)) <= TOL_BF16
    assert abs(float(lam.grad) - ref[5]) <= 2e-3 * max(1.0, abs(ref[5]))
