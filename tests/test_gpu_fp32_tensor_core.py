"""fp32 inputs at head_dim 64 and 128 on the tensor cores (three TF32 products
per fp32 product), through the C ABI: given the workspace that
``tda_workspace_size(.., TDA_F32, .., D, ..)`` reports, ``tda_rect_fwd`` /
``tda_diff_fwd`` take that path; without a workspace they run the exact-fp32
CUDA-core kernel.  Both are checked against the fp64 oracle at the fp32
tolerance (rel-L2 <= 1e-5) and against each other, on ragged lengths,
negative / zero / positive beta, the general power and both forms.
"""
import numpy as np
import pytest
import torch

from oracle import tda_oracle as O
from tda_b200 import _lib, ops

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL_F32 = 1e-5

CASES = [
    # (batch_heads, S, beta, p, normalize, differential, head_dim)
    (2, 1, 1.0, 2.0, True, False, 64),
    (2, 63, 1.0, 2.0, True, True, 64),
    (3, 200, -0.5, 2.0, True, False, 64),
    (1, 129, 0.0, 1.0, False, True, 64),
    (2, 300, 1.0, 1.5, False, False, 64),
    (1, 1000, 0.5, 3.0, True, True, 64),
    (4, 256, 2.0, 2.0, True, True, 64),
    (1, 777, -1.0, 1.0, True, True, 64),
    (2, 1, 1.0, 2.0, True, False, 128),
    (2, 95, 1.0, 2.0, True, True, 128),
    (3, 200, -0.5, 2.0, True, False, 128),
    (1, 129, 0.0, 1.0, False, True, 128),
    (2, 300, 1.0, 1.5, False, False, 128),
    (1, 1000, 0.5, 3.0, True, True, 128),
    (1, 777, -1.0, 1.0, True, True, 128),
]


def _run(lib, xs, BH, S, beta, lam, p, normalize, diff, with_ws):
    D = xs[0].shape[-1]
    out = torch.empty((BH, S, D), dtype=torch.float32, device=DEV)
    status = ops._status_word(torch.device(DEV))
    ws_n = lib.tda_workspace_size(int(diff), _lib.TDA_F32, BH, S, D, int(normalize)) if with_ws else 0
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    ptr = [x.data_ptr() for x in xs]
    if diff:
        rc = lib.tda_diff_fwd(*ptr, out.data_ptr(), _lib.TDA_F32, _lib.TDA_F32, BH, S, D, beta, lam, p,
                              int(normalize), ws.data_ptr() if ws_n else None, ws_n, status.data_ptr(), st)
    else:
        rc = lib.tda_rect_fwd(ptr[0], ptr[2], ptr[4], out.data_ptr(), _lib.TDA_F32, _lib.TDA_F32, BH, S, D, beta,
                              p, int(normalize), ws.data_ptr() if ws_n else None, ws_n, status.data_ptr(), st)
    _lib.check(rc)
    torch.cuda.synchronize()
    ops.check_status()
    return out.cpu().numpy()


def test_workspace_size_reports_the_split_copies():
    lib = _lib.load()
    BH, S = 3, 200
    rect = lib.tda_workspace_size(0, _lib.TDA_F32, BH, S, 64, 1)
    diff = lib.tda_workspace_size(1, _lib.TDA_F32, BH, S, 64, 0)
    # at least the high / low copies of q, k (per branch) and of v
    assert rect >= 6 * BH * S * 64 * 4 and diff >= 10 * BH * S * 64 * 4
    assert lib.tda_workspace_size(0, _lib.TDA_F32, BH, S, 128, 1) >= 6 * BH * S * 128 * 4
    assert lib.tda_workspace_size(0, _lib.TDA_F32, BH, S, 32, 1) == 0  # CUDA-core path, no workspace


@pytest.mark.parametrize("case", CASES, ids=[f"bh{c[0]}_S{c[1]}_b{c[2]}_p{c[3]}_n{int(c[4])}_d{int(c[5])}_D{c[6]}"
                                             for c in CASES])
def test_tensor_core_fp32_matches_oracle_and_cuda_core(case):
    BH, S, beta, p, normalize, diff, D = case
    lam = 0.6
    g = torch.Generator().manual_seed(BH * 1000 + S + D)
    xs_h = [torch.randn((BH, S, D), generator=g) * (1.0 if normalize else 2.0) for _ in range(5)]
    xs = [x.to(DEV) for x in xs_h]
    xn = [x.numpy()[None] for x in xs_h]
    if diff:
        ref = O.diff_fwd(*xn, beta, lam, p, normalize)[0]
    else:
        ref = O.rect_fwd(xn[0], xn[2], xn[4], beta, p, normalize)[0]
    lib = _lib.load()
    tc = _run(lib, xs, BH, S, beta, lam, p, normalize, diff, True)
    cc = _run(lib, xs, BH, S, beta, lam, p, normalize, diff, False)
    assert np.isfinite(tc).all()
    e_tc = O.rel_l2(tc, ref)
    e_cc = O.rel_l2(cc, ref)
    assert e_tc <= TOL_F32, f"tensor-core fp32 rel-L2 {e_tc:.3e}"
    assert e_cc <= TOL_F32, f"CUDA-core fp32 rel-L2 {e_cc:.3e}"
    assert O.rel_l2(tc, cc) <= 2 * TOL_F32


def test_public_api_fp32_head_dim_64_uses_workspace_path():
    """The public functions size the workspace from tda_workspace_size, so fp32
    at head_dim 64 reaches the tensor-core path; the result stays within the
    fp32 tolerance on a (batch, heads) layout with several heads."""
    g = torch.Generator().manual_seed(7)
    xs_h = [torch.randn((2, 3, 333, 64), generator=g) for _ in range(5)]
    xs = [x.to(DEV) for x in xs_h]
    xn = [x.numpy() for x in xs_h]
    out = ops.differential_threshold_rela_triton(*xs, torch.tensor(1.0), torch.tensor(0.5), 2.0, True)
    ref = O.diff_fwd(*xn, 1.0, 0.5, 2.0, True)
    assert out.dtype == torch.float32
    assert O.rel_l2(out.cpu().numpy(), ref) <= TOL_F32


def test_timeout_reports_status_and_context_survives():
    """Failure detection of the fp32 tensor-core kernel without a GPU fault:
    the test hook makes its producer skip the first Q load, every bounded wait
    gives up after 50 ms, the kernel frees its tensor memory and reports a
    status the host reads; the next call on the same context is correct."""
    lib = _lib.load()
    BH, S = 2, 300
    g = torch.Generator().manual_seed(21)
    xs_h = [torch.randn((BH, S, 64), generator=g) for _ in range(5)]
    xs = [x.to(DEV) for x in xs_h]
    lib.tda_debug_set(1, 50_000_000)
    try:
        with pytest.raises(_lib.TdaError, match="status"):
            _run(lib, xs, BH, S, 1.0, 0.5, 2.0, True, True, True)
    finally:
        lib.tda_debug_set(0, 0)
    ops.check_status()  # cleared by the failed check
    out = _run(lib, xs, BH, S, 1.0, 0.5, 2.0, True, True, True)
    ref = O.diff_fwd(*[x.numpy()[None] for x in xs_h], 1.0, 0.5, 2.0, True)[0]
    assert O.rel_l2(out, ref) <= TOL_F32


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("beta", [1.0, -0.5])
def test_long_sequence_sampled_rows(beta, D):
    """S = 4096 (64 or 128 key tiles accumulated per row): a sample of query
    rows at the start, middle and end against the oracle, differential form."""
    BH, S = 2, 4096
    g = torch.Generator().manual_seed(4096 + int(10 * beta) + D)
    xs_h = [torch.randn((BH, S, D), generator=g) for _ in range(5)]
    xs = [x.to(DEV) for x in xs_h]
    rows = list(range(0, 64)) + list(range(2000, 2064)) + list(range(S - 64, S))
    lib = _lib.load()
    out = _run(lib, xs, BH, S, beta, 0.5, 2.0, True, True, True)
    ref = O.diff_fwd(*[x.numpy()[None] for x in xs_h], beta, 0.5, 2.0, True, rows=rows)[0]
    assert O.rel_l2(out[:, rows], ref[:, rows]) <= TOL_F32


def test_public_api_fp32_strided_views():
    """(B, S, H, D) fp32 storage passed as (B, H, S, D) views: made contiguous by
    the public API, then the tensor-core fp32 path."""
    g = torch.Generator().manual_seed(31)
    xs_h = [torch.randn((1, 300, 3, 64), generator=g) for _ in range(3)]
    views = [x.to(DEV).transpose(1, 2) for x in xs_h]
    out = ops.threshold_rela_triton(*views, torch.tensor(1.0), 2.0, True)
    ref = O.rect_fwd(*[x.transpose(1, 2).contiguous().numpy() for x in xs_h], 1.0, 2.0, True)
    assert out.dtype == torch.float32 and out.shape == (1, 3, 300, 64)
    assert O.rel_l2(out.cpu().numpy(), ref) <= TOL_F32
