"""tda_diff_fwd_noalloc: the fused differential forward without any device
allocation.

Some callers cannot call cudaMalloc: code running inside an allocator or
memory-pool callback (allocating would re-enter the allocator), runtimes that
forbid allocation once they have started, and plugins whose host owns all
device memory and hands them only inputs and outputs.  For them the library
keeps the forward's scratch (the inverse key norms) in a fixed array of its
own instead of a caller-provided workspace.  These tests call that entry point
through the C ABI and compare it with the workspace-taking tda_diff_fwd and
with the fp64 oracle, on consecutive calls (the array keeps what the last call
wrote, so a later call must not depend on it), on the branches that need no
scratch (normalize = 0, fp32 inputs), and on a call that fills the array
exactly to its limit.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest
import torch

from oracle import tda_oracle as O
from tda_b200 import _lib

TOL = 1e-3      # the bf16-path tolerance used by the parity tests
TOL_F32 = 1e-5  # the fp32-path tolerance used by the parity tests
LIMIT_ROWS = 1 << 20  # batch_heads * round_up(seq_len, 128) the static scratch holds


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den else float(np.linalg.norm(a - b))


def test_noalloc_rejects_sizes_beyond_its_static_scratch():
    # checked on the host before any CUDA call: 1024 heads x 2048 rows > 2^20
    lib = _lib.load()
    rc = lib.tda_diff_fwd_noalloc(16, 16, 16, 16, 16, 16, _lib.TDA_BF16, _lib.TDA_BF16, 1024, 2048, 128,
                                  1.0, 0.5, 2.0, 1, 16, None)
    assert rc == _lib.TDA_ERR_INVALID
    assert b"static scratch" in lib.tda_last_error()
    # one 128-row tile past the limit is rejected as well
    rc = lib.tda_diff_fwd_noalloc(16, 16, 16, 16, 16, 16, _lib.TDA_BF16, _lib.TDA_BF16, 129, 8192, 64,
                                  1.0, 0.5, 2.0, 1, 16, None)
    assert rc == _lib.TDA_ERR_INVALID


def _call_both(lib, xs, BH, S, D, dtype, out_kind, out_dt, beta, lam, p, norm, status, stream):
    """The workspace entry point and the no-alloc one on the same inputs;
    returns (workspace output, no-alloc output)."""
    dev = xs[0].device
    ptrs = [x.data_ptr() for x in xs]
    ref = torch.empty(BH, S, D, dtype=out_dt, device=dev)
    new = torch.full_like(ref, float("nan"))
    ws_n = lib.tda_workspace_size(1, dtype, BH, S, D, int(norm))
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)
    rc = lib.tda_diff_fwd(*ptrs, ref.data_ptr(), dtype, out_kind, BH, S, D, beta, lam, p, int(norm),
                          ws.data_ptr() if ws_n else None, ws_n, status.data_ptr(), stream)
    assert rc == _lib.TDA_OK, lib.tda_last_error()
    rc = lib.tda_diff_fwd_noalloc(*ptrs, new.data_ptr(), dtype, out_kind, BH, S, D, beta, lam, p, int(norm),
                                  status.data_ptr(), stream)
    assert rc == _lib.TDA_OK, lib.tda_last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return ref, new


def _oracle_rows(xs, bhs, rows, beta, lam, p, norm):
    """fp64 oracle of the differential form on heads ``bhs`` and ``rows``."""
    out = []
    for b in bhs:
        a = [x[b].float().cpu().numpy()[None, None] for x in xs]
        out.append(O.diff_fwd(*a, beta, lam, p, norm, rows=rows)[0, 0, rows])
    return np.stack(out)


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_and_oracle_on_consecutive_calls():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    # consecutive calls with different inputs, sizes and branches: none may be
    # affected by what an earlier call left in the shared scratch
    cases = [
        # BH, S, D, seed, dtype, normalize, beta
        (4, 700, 128, 1, torch.bfloat16, True, 0.3),
        (3, 260, 64, 2, torch.bfloat16, True, -0.4),
        (2, 300, 128, 3, torch.bfloat16, False, 0.5),  # no scratch needed: forwards to tda_diff_fwd
        (2, 200, 64, 4, torch.float32, True, 0.3),     # fp32: the CUDA-core kernel, no scratch
        (4, 700, 128, 5, torch.bfloat16, True, 1.0),   # same size as the first call, new data
    ]
    lam, p = 0.5, 2.0
    for BH, S, D, seed, dt, norm, beta in cases:
        g = torch.Generator().manual_seed(seed)
        xs = [torch.randn(BH, S, D, generator=g).to(dt).to(dev) for _ in range(5)]
        kind = _lib.TDA_F32 if dt == torch.float32 else _lib.TDA_BF16
        outs = ((_lib.TDA_F32, torch.float32),) if dt == torch.float32 else \
            ((_lib.TDA_F32, torch.float32), (_lib.TDA_BF16, torch.bfloat16))
        rows = np.unique(np.concatenate([np.arange(8), np.linspace(8, S - 1, 40).astype(int)]))
        want = _oracle_rows(xs, [0, BH - 1], rows, beta, lam, p, norm)
        for out_kind, out_dt in outs:
            ref, new = _call_both(lib, xs, BH, S, D, kind, out_kind, out_dt, beta, lam, p, norm, status, stream)
            assert torch.isfinite(new).all()
            assert ref.abs().sum() > 0
            tol = TOL_F32 if dt == torch.float32 else TOL
            assert _rel(new, ref) <= tol, (BH, S, D, dt, norm)
            got = new[[0, BH - 1]][:, torch.as_tensor(rows, device=dev)].float().cpu().numpy()
            if out_dt == torch.bfloat16:
                assert O.rel_l2(got, O.bf16_round(want)) <= TOL, (BH, S, D, dt, norm)
            else:
                assert O.rel_l2(got, want) <= tol, (BH, S, D, dt, norm)


@pytest.mark.gpu
def test_noalloc_at_its_size_limit():
    """batch_heads * round_up(seq_len, 128) equal to the limit: k2's key table
    ends exactly at the end of the static array."""
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    BH, S, D = 128, 8192, 64
    assert BH * S == LIMIT_ROWS
    xs = []
    for t in range(5):
        g = torch.Generator(device=dev).manual_seed(900 + t)
        xs.append(torch.randn(BH, S, D, generator=g, device=dev).to(torch.bfloat16))
    for _ in range(2):  # two calls in a row on the full array
        ref, new = _call_both(lib, xs, BH, S, D, _lib.TDA_BF16, _lib.TDA_F32, torch.float32, 1.0, 0.5, 2.0, True,
                              status, stream)
        assert torch.isfinite(new).all()
        assert _rel(new, ref) <= TOL
    rows = np.unique(np.concatenate([np.arange(16), np.arange(S - 16, S), np.linspace(16, S - 17, 32).astype(int)]))
    want = _oracle_rows(xs, [0, BH - 1], rows, 1.0, 0.5, 2.0, True)
    got = new[[0, BH - 1]][:, torch.as_tensor(rows, device=dev)].cpu().numpy()
    assert O.rel_l2(got, want) <= TOL
