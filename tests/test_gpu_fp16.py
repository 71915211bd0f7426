"""fp16 inputs on the tcgen05 tensor cores (kind::f16 with fp16 operands).

The reference accepts any float dtype: it upcasts to fp32 and casts the
output back to q's dtype (triton_threshold_attention.py:356-360, :392-393).
Here normalized fp16 inputs at head_dim 64 / 128 stay fp16 on the tensor
cores: QK^T in fp16 x fp16 -> fp32, P written as fp16 hi + lo of a
power-of-two-scaled P (P is bounded when q, k are normalized), fp16 output.
Unnormalized fp16 inputs (P unbounded) are widened to fp32 instead.

Tolerances (rel-L2), as for bf16: the fp32 accumulator output vs the fp64
oracle <= 1e-3 and the fp16 output vs the fp16-rounded oracle <= 1e-3.
"""
import zlib

import numpy as np
import pytest
import torch

import tda_b200
from oracle import tda_oracle as O
from tda_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 1e-3


def _gen(seed, shape, n=5, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(shape, generator=g) * std).to(torch.float16) for _ in range(n)]


def _np(t):
    return t.float().cpu().numpy()


def _f16_round(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def _check(acc, out, ref):
    assert out.dtype == torch.float16
    e_acc = O.rel_l2(_np(acc), ref)
    e_out = O.rel_l2(_np(out), _f16_round(ref))
    assert e_acc <= TOL, f"fp32 accumulator rel-L2 {e_acc:.3e}"
    assert e_out <= TOL, f"fp16 output rel-L2 vs fp16(oracle) {e_out:.3e}"
    return e_acc


CASES = [((1, 2, 300, 64), 1.0, 2.0), ((2, 3, 520, 128), 1.0, 2.0), ((1, 2, 257, 128), 0.0, 2.0),
         ((1, 2, 300, 128), -0.5, 2.0), ((1, 2, 200, 64), 0.5, 3.0), ((1, 2, 200, 128), 1.0, 1.0),
         ((1, 2, 260, 64), 0.5, 1.5), ((1, 1, 1, 128), 1.0, 2.0)]


@pytest.mark.parametrize("shape,beta,p", CASES, ids=[f"{s}-b{b}-p{p}" for s, b, p in CASES])
@pytest.mark.parametrize("op", ["rect", "diff"])
def test_fp16_tensor_core_matches_oracle(shape, beta, p, op):
    xs = _gen(zlib.crc32(repr((shape, beta, p, op)).encode()) % 1000, shape)
    xn = [_np(x) for x in xs]
    dev = [x.to(DEV) for x in xs]
    lam = 0.6
    if op == "rect":
        ref = O.rect_fwd(xn[0], xn[2], xn[4], beta, p, True)
        acc = tda_b200.rect_forward(dev[0], dev[2], dev[4], beta, p, True, out_dtype=torch.float32)
        out = tda_b200.threshold_rela_triton(dev[0], dev[2], dev[4], torch.tensor(beta), p, True)
    else:
        ref = O.diff_fwd(*xn, beta, lam, p, True)
        acc = tda_b200.diff_forward(*dev, beta, lam, p, True, out_dtype=torch.float32)
        out = tda_b200.differential_threshold_rela_triton(*dev, torch.tensor(beta), torch.tensor(lam), p, True)
    e = _check(acc, out, ref)
    # hi + lo P on fp16 operands is far inside the gate
    assert e <= 2e-4, e
    tda_b200.check_status()


def test_fp16_larger_and_per_head_lambda():
    B, H, S, D = 2, 4, 2048, 128
    xs = _gen(7, (B, H, S, D))
    xn = [_np(x) for x in xs]
    dev = [x.to(DEV) for x in xs]
    lam = torch.tensor([0.2, 0.5, 0.8, 1.0]).view(1, H, 1, 1)
    acc = tda_b200.diff_forward(*dev, 1.0, lam.to(DEV), 2.0, True, out_dtype=torch.float32)
    out = tda_b200.differential_threshold_rela_triton(*dev, 1.0, lam.to(DEV), 2.0, True)
    rows = np.unique(np.concatenate([np.arange(64), np.arange(S - 64, S), np.linspace(64, S - 65, 64).astype(int)]))
    for b, h in ((0, 0), (1, 3), (0, 2)):
        sl = [x[b:b + 1, h:h + 1] for x in xn]
        ref = O.diff_fwd(*sl, 1.0, float(lam[0, h]), 2.0, True, rows=rows)[0, 0, rows]
        assert O.rel_l2(_np(acc[b, h, rows]), ref) <= TOL
        assert O.rel_l2(_np(out[b, h, rows]), _f16_round(ref)) <= TOL
    tda_b200.check_status()


def test_fp16_unnormalized_widens_to_fp32():
    # raw scores are unbounded without normalize: the fp32 path runs, output fp16
    xs = _gen(9, (1, 2, 150, 64), std=0.5)
    xn = [_np(x) for x in xs]
    out = tda_b200.threshold_rela_triton(*[x.to(DEV) for x in xs[:3]], 1.0, 2.0, False)
    assert out.dtype == torch.float16
    ref = O.rect_fwd(xn[0], xn[1], xn[2], 1.0, 2.0, False)
    assert O.rel_l2(_np(out), _f16_round(ref)) <= TOL


def test_fp16_through_no_alloc_entry_point():
    lib = _lib.load()
    BH, S, D = 3, 400, 128
    xs = [x.view(BH, S, D).to(DEV) for x in _gen(11, (1, BH, S, D))]
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.empty(BH, S, D, dtype=torch.float32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.tda_diff_fwd_noalloc(*[x.data_ptr() for x in xs], out.data_ptr(), _lib.TDA_F16, _lib.TDA_F32, BH, S, D,
                                  1.0, 0.5, 2.0, 1, status.data_ptr(), stream)
    assert rc == _lib.TDA_OK, lib.tda_last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = O.diff_fwd(*[_np(x)[None] for x in xs], 1.0, 0.5, 2.0, True)[0]
    assert O.rel_l2(_np(out), ref) <= TOL
