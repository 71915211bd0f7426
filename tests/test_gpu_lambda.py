"""lambda as a device tensor in the differential form (reference :516-517,
out1 - clamp(lambda, 0, 1) * out2, lambda broadcast against the output).

A lambda that varies at most over (batch, head) -- a 0-dim CUDA scalar, per
head, per (batch, head) -- is read by the fused kernel itself through
tda_diff_fwd_lambda: one pass, no host synchronisation.  Every case is checked
against the fp64 oracle applied head by head with that head's lambda, on the
bf16 tensor-core path, the fp32 tensor-core and CUDA-core paths, and strided
(B, S, H, D) views.  A lambda that also varies along the sequence falls back
to two passes and the reference's combine.
"""
import numpy as np
import pytest
import torch

import tda_b200
from oracle import tda_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL_BF16 = 1e-3
TOL_F32 = 1e-5


def _gen(seed, shape, dtype=torch.bfloat16, n=5):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(shape, generator=g).to(dtype) for _ in range(n)]


def _np(t):
    return t.float().cpu().numpy()


def _oracle_per_head(xn, lam4, beta, p, norm):
    """Oracle with lambda taken per (batch, head) from a (B|1, H|1, 1, 1) array."""
    B, H = xn[0].shape[:2]
    out = np.zeros(xn[0].shape, dtype=np.float64)
    for b in range(B):
        for h in range(H):
            lam = float(lam4[b if lam4.shape[0] > 1 else 0, h if lam4.shape[1] > 1 else 0, 0, 0])
            out[b, h] = O.diff_fwd(*[x[b:b + 1, h:h + 1] for x in xn], beta, lam, p, norm)[0, 0]
    return out


LAMS = {
    "scalar_0d": lambda B, H: torch.tensor(0.35),
    "per_head": lambda B, H: torch.tensor([0.2, 0.9, -0.3, 1.4][:H]).view(1, H, 1, 1),
    "per_head_3d": lambda B, H: torch.tensor([0.6, 0.1, 0.75, 0.5][:H]).view(H, 1, 1),
    "per_batch_head": lambda B, H: torch.linspace(-0.2, 1.2, B * H).view(B, H, 1, 1),
}


@pytest.mark.parametrize("lam_name", list(LAMS))
@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.bfloat16, 64), (torch.float32, 64),
                                     (torch.float32, 32)])
def test_device_lambda_matches_oracle(lam_name, dtype, D):
    B, H, S = 2, 4, 300
    xs = _gen(31 + D, (B, H, S, D), dtype)
    xn = [_np(x) for x in xs]
    lam = LAMS[lam_name](B, H)
    lam_cuda = lam.to(DEV)
    beta, p = 0.5, 2.0
    dev = [x.to(DEV) for x in xs]
    lam4 = lam.reshape((1,) * (4 - lam.dim()) + tuple(lam.shape)).numpy()
    ref = _oracle_per_head(xn, lam4, beta, p, True)
    if dtype == torch.float32:
        out = tda_b200.differential_threshold_rela_triton(*dev, torch.tensor(beta), lam_cuda, p, True)
        assert out.dtype == torch.float32
        assert O.rel_l2(_np(out), ref) <= TOL_F32
    else:
        acc = tda_b200.diff_forward(*dev, beta, lam_cuda, p, True, out_dtype=torch.float32)
        out = tda_b200.differential_threshold_rela_triton(*dev, torch.tensor(beta), lam_cuda, p, True)
        assert out.dtype == torch.bfloat16
        assert O.rel_l2(_np(acc), ref) <= TOL_BF16
        assert O.rel_l2(_np(out), O.bf16_round(ref)) <= TOL_BF16
    tda_b200.check_status()


@pytest.mark.parametrize("p", [1.0, 3.0, 1.5])
def test_device_lambda_powers_and_beta_neg(p):
    # lambda folded into the second branch as lambda^(1/p) (p = 1, 3) and the
    # general power's explicit weight (p = 1.5); beta < 0 processes every tile
    B, H, S, D = 1, 3, 260, 128
    xs = _gen(41, (B, H, S, D))
    xn = [_np(x) for x in xs]
    lam = torch.tensor([0.3, 0.8, 0.55]).view(1, H, 1, 1)
    for beta in (1.0, -0.5):
        acc = tda_b200.diff_forward(*[x.to(DEV) for x in xs], beta, lam.to(DEV), p, True, out_dtype=torch.float32)
        ref = _oracle_per_head(xn, lam.numpy(), beta, p, True)
        assert O.rel_l2(_np(acc), ref) <= TOL_BF16, (p, beta)
    tda_b200.check_status()


def test_device_lambda_strided_views():
    # (B, S, H, D) storage read in place through the strided entry, per-head lambda
    B, H, S, D = 2, 3, 200, 128
    st = _gen(43, (B, S, H, D))
    views = [x.to(DEV).transpose(1, 2) for x in st]
    lam = torch.tensor([0.1, 0.5, 0.9]).view(1, H, 1, 1)
    acc = tda_b200.diff_forward(*views, 1.0, lam.to(DEV), 2.0, True, out_dtype=torch.float32)
    ref = _oracle_per_head([_np(v.contiguous()) for v in views], lam.numpy(), 1.0, 2.0, True)
    assert O.rel_l2(_np(acc), ref) <= TOL_BF16
    tda_b200.check_status()


def test_device_scalar_lambda_equals_host_scalar():
    # a 0-dim CUDA lambda runs the device path; the host float the scalar
    # path: the same arithmetic (lambda^(1/2) formed on either side)
    xs = [x.to(DEV) for x in _gen(44, (1, 2, 384, 128))]
    a = tda_b200.diff_forward(*xs, 1.0, torch.tensor(0.5, device=DEV), 2.0, True, out_dtype=torch.float32)
    b = tda_b200.diff_forward(*xs, 1.0, 0.5, 2.0, True, out_dtype=torch.float32)
    assert O.rel_l2(_np(a), _np(b)) <= 1e-6


def test_lambda_varying_along_sequence_falls_back_to_combine():
    B, H, S, D = 1, 2, 150, 64
    xs = _gen(45, (B, H, S, D))
    xn = [_np(x) for x in xs]
    lam = torch.linspace(0.0, 1.0, S).view(1, 1, S, 1)
    out = tda_b200.diff_forward(*[x.to(DEV) for x in xs], 1.0, lam.to(DEV), 2.0, True, out_dtype=torch.float32)
    o1 = O.rect_fwd(xn[0], xn[2], xn[4], 1.0, 2.0, True)
    o2 = O.rect_fwd(xn[1], xn[3], xn[4], 1.0, 2.0, True)
    ref = o1 - lam.double().numpy() * o2
    assert O.rel_l2(_np(out), ref) <= TOL_BF16


def test_device_lambda_is_graph_capturable():
    """No host synchronisation on the device-lambda path: the public call can
    be captured into a CUDA graph (a host read of lambda would fail the
    capture) and its replays follow lambda's current device value."""
    xs = [x.to(DEV) for x in _gen(46, (1, 4, 256, 128))]
    lam = torch.tensor([0.25, 0.5, 0.75, 1.0], device=DEV).view(1, 4, 1, 1)
    beta = 1.0
    tda_b200.diff_forward(*xs, beta, lam, 2.0, True)  # warm-up (status word, kernel attributes)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            out = tda_b200.diff_forward(*xs, beta, lam, 2.0, True, out_dtype=torch.float32)
    for vals in ([0.25, 0.5, 0.75, 1.0], [0.9, 0.0, 0.3, 0.6]):
        lam.copy_(torch.tensor(vals, device=DEV).view(1, 4, 1, 1))
        g.replay()
        torch.cuda.synchronize()
        eager = tda_b200.diff_forward(*xs, beta, lam, 2.0, True, out_dtype=torch.float32)
        assert torch.equal(out, eager)
    tda_b200.check_status()

