"""Parity of the CUDA path (through the public API -> C ABI) against the CPU
oracle, which is itself pinned to the reference's outputs
(tests/test_oracle_golden.py).

Tolerances (rel-L2 over the compared entries):
  * fp32 inputs (exact-fp32 kernel):            <= 1e-5 vs the fp64 oracle.
  * bf16 inputs (tcgen05 kernel):
      - fp32 accumulator output vs the oracle:  <= 1e-3
      - bf16 output vs the bf16-rounded oracle: <= 1e-3
    (rounding the exact result to bf16 alone gives ~1.7e-3, so a bf16 output
    cannot be compared with the unrounded oracle at 1e-3.)
"""
import zlib

import numpy as np
import pytest
import torch

import tda_b200
from golden_io import load_cases
from oracle import tda_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL_F32 = 1e-5
TOL_BF16 = 1e-3


def _t(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(DEV).to(dtype)


def _np(t):
    return t.float().cpu().numpy()


def _gen(seed, n, shape, std=1.0, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return [(torch.randn(shape, generator=g) * std).to(dtype) for _ in range(n)]


def _check_bf16(acc32, out16, ref):
    e_acc = O.rel_l2(acc32, ref)
    e_out = O.rel_l2(out16, O.bf16_round(ref))
    assert e_acc <= TOL_BF16, f"fp32 accumulator rel-L2 {e_acc:.3e}"
    assert e_out <= TOL_BF16, f"bf16 output rel-L2 vs bf16(oracle) {e_out:.3e}"
    return e_acc, e_out


# ----------------------------------------------------------------- golden cases
CASES = load_cases()


@pytest.mark.parametrize("case", [c for c in CASES if c[0]["dtype"] == "f32"],
                         ids=[c[0]["name"] for c in CASES if c[0]["dtype"] == "f32"])
def test_golden_fp32(case):
    """fp32 golden inputs through the fp32 kernel vs the reference's outputs."""
    m, a = case
    beta = torch.tensor(m["beta"])
    if m["op"] == "rect":
        out = tda_b200.threshold_rela_triton(_t(a["q"], torch.float32), _t(a["k"], torch.float32),
                                             _t(a["v"], torch.float32), beta, m["p"], m["normalize"])
    else:
        t = [_t(a[n], torch.float32) for n in ("q1", "q2", "k1", "k2", "v")]
        out = tda_b200.differential_threshold_rela_triton(*t, beta, torch.tensor(m["lam"]), m["p"], m["normalize"])
    assert out.dtype == torch.float32 and out.shape == tuple(m["shape"])
    assert O.rel_l2(_np(out), a["out"]) <= TOL_F32


@pytest.mark.parametrize("case", CASES, ids=[c[0]["name"] for c in CASES])
def test_golden_bf16_tensor_core(case):
    """Golden inputs rounded to bf16 through the tensor-core kernel (D = 64/128)
    or the widened fp32 kernel (other D), vs the oracle on the same inputs."""
    m, a = case
    names = ("q", "k", "v") if m["op"] == "rect" else ("q1", "q2", "k1", "k2", "v")
    xs = {n: O.bf16_round(a[n]) for n in names}
    beta = torch.tensor(m["beta"])
    if m["op"] == "rect":
        args = [_t(xs[n], torch.bfloat16) for n in names]
        ref = O.rect_fwd(xs["q"], xs["k"], xs["v"], m["beta"], m["p"], m["normalize"])
        acc = tda_b200.rect_forward(*args, beta, m["p"], m["normalize"], out_dtype=torch.float32)
        out = tda_b200.threshold_rela_triton(*args, beta, m["p"], m["normalize"])
    else:
        args = [_t(xs[n], torch.bfloat16) for n in names]
        ref = O.diff_fwd(xs["q1"], xs["q2"], xs["k1"], xs["k2"], xs["v"], m["beta"], m["lam"], m["p"],
                         m["normalize"])
        lam = torch.tensor(m["lam"])
        acc = tda_b200.diff_forward(*args, beta, lam, m["p"], m["normalize"], out_dtype=torch.float32)
        out = tda_b200.differential_threshold_rela_triton(*args, beta, lam, m["p"], m["normalize"])
    assert out.dtype == torch.bfloat16
    _check_bf16(_np(acc), _np(out), ref)
    tda_b200.check_status()


# ------------------------------------------------------------ seeded sweeps
SHAPES = [(1, 2, 128, 64), (1, 2, 256, 128), (2, 1, 100, 64), (1, 1, 1, 128), (1, 2, 129, 128),
          (1, 1, 383, 64), (1, 1, 640, 128)]


@pytest.mark.parametrize("shape", SHAPES, ids=[str(s) for s in SHAPES])
@pytest.mark.parametrize("normalize", [True, False])
@pytest.mark.parametrize("op", ["rect", "diff"])
def test_bf16_shapes(shape, normalize, op):
    beta, p, lam = 1.0, 2.0, 0.5
    xs = _gen(zlib.crc32(repr((shape, normalize, op)).encode()) & 0xFFFF, 5, shape)
    xn = [_np(x) for x in xs]
    dev = [x.to(DEV) for x in xs]
    if op == "rect":
        ref = O.rect_fwd(xn[0], xn[2], xn[4], beta, p, normalize)
        acc = tda_b200.rect_forward(dev[0], dev[2], dev[4], beta, p, normalize, out_dtype=torch.float32)
        out = tda_b200.threshold_rela_triton(dev[0], dev[2], dev[4], torch.tensor(beta), p, normalize)
    else:
        ref = O.diff_fwd(xn[0], xn[1], xn[2], xn[3], xn[4], beta, lam, p, normalize)
        acc = tda_b200.diff_forward(*dev, beta, lam, p, normalize, out_dtype=torch.float32)
        out = tda_b200.differential_threshold_rela_triton(*dev, torch.tensor(beta), torch.tensor(lam), p, normalize)
    _check_bf16(_np(acc), _np(out), ref)
    tda_b200.check_status()


PARAMS = [(0.5, 1.0), (1.0, 3.0), (2.0, 1.5), (0.0, 2.0), (-0.5, 2.0), (-1.0, 1.0), (1.0, 2.0)]


@pytest.mark.parametrize("beta,p", PARAMS, ids=[f"b{b}_p{p}" for b, p in PARAMS])
@pytest.mark.parametrize("normalize", [True, False])
@pytest.mark.parametrize("D", [64, 128])
def test_bf16_params(beta, p, normalize, D):
    shape = (1, 2, 300, D)
    xs = _gen(17 + D, 5, shape, std=2.0 if not normalize else 1.0)
    xn = [_np(x) for x in xs]
    dev = [x.to(DEV) for x in xs]
    lam = 0.7
    ref_r = O.rect_fwd(xn[0], xn[2], xn[4], beta, p, normalize)
    acc_r = tda_b200.rect_forward(dev[0], dev[2], dev[4], beta, p, normalize, out_dtype=torch.float32)
    out_r = tda_b200.threshold_rela_triton(dev[0], dev[2], dev[4], beta, p, normalize)
    _check_bf16(_np(acc_r), _np(out_r), ref_r)
    ref_d = O.diff_fwd(*xn, beta, lam, p, normalize)
    acc_d = tda_b200.diff_forward(*dev, beta, lam, p, normalize, out_dtype=torch.float32)
    out_d = tda_b200.differential_threshold_rela_triton(*dev, beta, torch.tensor(lam), p, normalize)
    _check_bf16(_np(acc_d), _np(out_d), ref_d)
    tda_b200.check_status()


@pytest.mark.parametrize("beta,p", PARAMS, ids=[f"b{b}_p{p}" for b, p in PARAMS])
@pytest.mark.parametrize("D", [16, 64, 128, 256])
def test_fp32_params(beta, p, D):
    shape = (1, 2, 150, D)
    xs = _gen(99 + D, 5, shape, dtype=torch.float32)
    xn = [_np(x) for x in xs]
    dev = [x.to(DEV) for x in xs]
    for normalize in (True, False):
        ref = O.diff_fwd(*xn, beta, 0.4, p, normalize)
        out = tda_b200.differential_threshold_rela_triton(*dev, beta, torch.tensor(0.4), p, normalize)
        assert out.dtype == torch.float32
        assert O.rel_l2(_np(out), ref) <= TOL_F32
        ref = O.rect_fwd(xn[0], xn[2], xn[4], beta, p, normalize)
        out = tda_b200.threshold_rela_triton(dev[0], dev[2], dev[4], beta, p, normalize)
        assert O.rel_l2(_np(out), ref) <= TOL_F32


def test_other_dtypes_and_head_dims_widen_on_device():
    # fp16 inputs and bf16 with head_dim 32 go through the fp32 kernel; the
    # output keeps the input dtype (reference :392-393)
    for dtype, D in ((torch.float16, 64), (torch.bfloat16, 32)):
        xs = _gen(5, 3, (1, 2, 96, D), dtype=dtype)
        xn = [_np(x) for x in xs]
        out = tda_b200.threshold_rela_triton(*[x.to(DEV) for x in xs], torch.tensor(1.0), 2.0, True)
        assert out.dtype == dtype
        ref = torch.from_numpy(O.rect_fwd(*xn, 1.0, 2.0, True).astype(np.float32)).to(dtype).float().numpy()
        assert O.rel_l2(_np(out), ref) <= TOL_BF16


def test_lambda_clamp_and_broadcast():
    xs = [x.to(DEV) for x in _gen(3, 5, (2, 2, 130, 64))]
    xn = [_np(x) for x in xs]
    for lam in (-0.3, 0.0, 1.0, 1.7):
        ref = O.diff_fwd(*xn, 1.0, lam, 2.0, True)
        acc = tda_b200.diff_forward(*xs, 1.0, lam, 2.0, True, out_dtype=torch.float32)
        assert O.rel_l2(_np(acc), ref) <= TOL_BF16
    # per-head lambda (broadcast like the reference's out1 - lambda * out2)
    lam = torch.tensor([0.2, 0.9]).view(1, 2, 1, 1)
    out = tda_b200.differential_threshold_rela_triton(*xs, torch.tensor(1.0), lam, 2.0, True)
    ref = np.concatenate([O.diff_fwd(*[x[:, h:h + 1] for x in xn], 1.0, float(lam.view(-1)[h]), 2.0, True)
                          for h in range(2)], axis=1)
    assert O.rel_l2(_np(out), O.bf16_round(ref)) <= TOL_BF16


# --------------------------------------------------------- properties
def test_causality_bitwise():
    """Changing keys after row r leaves rows <= r bit-identical (masked scores
    are zeroed before the threshold, so key values there never matter)."""
    S, r = 700, 300
    xs = [x.to(DEV) for x in _gen(11, 5, (1, 2, S, 128))]
    base = tda_b200.diff_forward(*xs, 1.0, 0.5, 2.0, True, out_dtype=torch.float32)
    k1 = xs[2].clone()
    k2 = xs[3].clone()
    k1[:, :, r + 1:] = torch.randn_like(k1[:, :, r + 1:])
    k2[:, :, r + 1:] = torch.randn_like(k2[:, :, r + 1:])
    pert = tda_b200.diff_forward(xs[0], xs[1], k1, k2, xs[4], 1.0, 0.5, 2.0, True, out_dtype=torch.float32)
    assert torch.equal(base[:, :, :r + 1], pert[:, :, :r + 1])
    assert not torch.equal(base[:, :, r + 1:], pert[:, :, r + 1:])


def test_heads_independent_bitwise():
    """A (batch, head) slice computed alone equals the same slice of a batched
    call: the property the multi-GPU (batch x head) sharding relies on."""
    xs = [x.to(DEV) for x in _gen(12, 5, (2, 3, 257, 128))]
    full = tda_b200.diff_forward(*xs, 1.0, 0.5, 2.0, True)
    part = tda_b200.diff_forward(*[x[1:2, 1:3].contiguous() for x in xs], 1.0, 0.5, 2.0, True)
    assert torch.equal(full[1:2, 1:3], part)


def test_linearity_in_v():
    # small-integer V so that v1 + 2 v2 is exact in bf16
    g = torch.Generator().manual_seed(13)
    q1, q2, k1, k2 = [x.to(DEV) for x in _gen(13, 4, (1, 2, 512, 64))]
    v1, v2 = [torch.randint(-8, 9, (1, 2, 512, 64), generator=g).to(torch.bfloat16).to(DEV) for _ in range(2)]
    o1 = tda_b200.diff_forward(q1, q2, k1, k2, v1, 0.5, 0.5, 2.0, True, out_dtype=torch.float32)
    o2 = tda_b200.diff_forward(q1, q2, k1, k2, v2, 0.5, 0.5, 2.0, True, out_dtype=torch.float32)
    o12 = tda_b200.diff_forward(q1, q2, k1, k2, v1 + 2 * v2, 0.5, 0.5, 2.0, True, out_dtype=torch.float32)
    assert O.rel_l2(_np(o12), _np(o1 + 2 * o2)) <= 1e-5


def test_diff_lambda_zero_equals_rect():
    xs = [x.to(DEV) for x in _gen(14, 5, (1, 2, 384, 128))]
    d = tda_b200.diff_forward(*xs, 1.0, 0.0, 2.0, True, out_dtype=torch.float32)
    r = tda_b200.rect_forward(xs[0], xs[2], xs[4], 1.0, 2.0, True, out_dtype=torch.float32)
    assert O.rel_l2(_np(d), _np(r)) <= 1e-6


# ------------------------------------------------------- API behaviour
def test_errors_and_autograd():
    q = torch.randn(1, 2, 64, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        tda_b200.threshold_rela_triton(q, q[:, :, :32], q, 1.0)
    with pytest.raises(ValueError):
        x = torch.randn(1, 2, 64, 48, device=DEV)
        tda_b200.threshold_rela_triton(x, x, x, 1.0)
    qg = q.clone().requires_grad_(True)
    out = tda_b200.threshold_rela_triton(qg, q, q, torch.tensor(1.0), 2.0)
    assert out.requires_grad
    out.float().sum().backward()
    assert qg.grad is not None and qg.grad.shape == q.shape and qg.grad.dtype == q.dtype
    # head_dim 512 is outside the supported range and says so
    with pytest.raises(ValueError, match="head_dim"):
        x = torch.randn(1, 1, 32, 512, device=DEV)
        tda_b200.threshold_rela_triton(x, x, x, 1.0)
    empty = torch.zeros(1, 2, 0, 64, device=DEV, dtype=torch.bfloat16)
    assert tda_b200.threshold_rela_triton(empty, empty, empty, 1.0).shape == empty.shape


def test_noncontiguous_inputs_are_handled():
    # (B, S, H, D).transpose(1, 2) views: the reference indexes them wrongly;
    # here they are made contiguous first and give the right answer.
    xs = [x.to(DEV) for x in _gen(15, 3, (1, 200, 2, 64))]
    views = [x.transpose(1, 2) for x in xs]
    out = tda_b200.rect_forward(*views, 1.0, 2.0, True, out_dtype=torch.float32)
    ref = O.rect_fwd(*[_np(v.contiguous()) for v in views], 1.0, 2.0, True)
    assert O.rel_l2(_np(out), ref) <= TOL_BF16


def test_timeout_reports_status_and_context_survives():
    """Failure detection without a GPU fault: the test hook makes the kernel's
    producer skip the Q load, every bounded wait gives up after 50 ms, the
    kernel exits cleanly and reports a status the host reads; afterwards the
    context still works."""
    from tda_b200 import _lib
    lib = _lib.load()
    xs = [x.to(DEV) for x in _gen(16, 5, (1, 1, 256, 128))]
    lib.tda_debug_set(1, 50_000_000)
    try:
        tda_b200.diff_forward(*xs, 1.0, 0.5, 2.0, True)
        torch.cuda.synchronize()
    finally:
        lib.tda_debug_set(0, 0)
    with pytest.raises(_lib.TdaError, match="status"):
        tda_b200.check_status()
    tda_b200.check_status()  # cleared
    acc = tda_b200.diff_forward(*xs, 1.0, 0.5, 2.0, True, out_dtype=torch.float32)
    ref = O.diff_fwd(*[_np(x) for x in xs], 1.0, 0.5, 2.0, True)
    assert O.rel_l2(_np(acc), ref) <= TOL_BF16
    tda_b200.check_status()
