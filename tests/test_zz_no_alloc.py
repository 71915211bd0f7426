"""tda_diff_fwd_noalloc: the fused differential forward without any device
allocation.

Some callers cannot call cudaMalloc: code running inside an allocator or
memory-pool callback (allocating would re-enter the allocator), runtimes that
forbid allocation once they have started, and plugins whose host owns all
device memory and hands them only inputs and outputs.  For them the library
keeps the forward's scratch (the inverse key norms) in a fixed array of its
own instead of a caller-provided workspace.  These tests call that entry point
through the C ABI and compare it with the workspace-taking tda_diff_fwd.

This file is collected last on purpose, so a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest
import torch

from tda_b200 import _lib

TOL = 1e-3  # the bf16-path tolerance used by the parity tests


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


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    # two calls in a row with different inputs and sizes: the second call must
    # not be affected by what the first left in the shared scratch
    for BH, S, D, seed in ((4, 700, 128, 1), (3, 260, 64, 2)):
        g = torch.Generator().manual_seed(seed)
        xs = [torch.randn(BH, S, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(5)]
        ptrs = [x.data_ptr() for x in xs]
        for out_kind, out_dt in ((_lib.TDA_F32, torch.float32), (_lib.TDA_BF16, torch.bfloat16)):
            ref = torch.empty(BH, S, D, dtype=out_dt, device=dev)
            new = torch.full_like(ref, float("nan"))
            ws_n = lib.tda_workspace_size(1, _lib.TDA_BF16, BH, S, D, 1)
            ws = torch.empty(ws_n, dtype=torch.uint8, device=dev)
            rc = lib.tda_diff_fwd(*ptrs, ref.data_ptr(), _lib.TDA_BF16, out_kind, BH, S, D, 0.3, 0.5, 2.0, 1,
                                  ws.data_ptr(), ws_n, status.data_ptr(), stream)
            assert rc == _lib.TDA_OK, lib.tda_last_error()
            rc = lib.tda_diff_fwd_noalloc(*ptrs, new.data_ptr(), _lib.TDA_BF16, out_kind, BH, S, D, 0.3, 0.5, 2.0,
                                          1, status.data_ptr(), stream)
            assert rc == _lib.TDA_OK, lib.tda_last_error()
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert torch.isfinite(new).all()
            assert ref.abs().sum() > 0
            assert _rel(new, ref) <= TOL
