"""Strided (batch, heads, seq, dim) views on the tensor-core forward (row f3 of
the scope: general layouts through TMA descriptors).  The kernel reads such
views in place, so its output must equal, bit for bit, the output for the same
values made contiguous; views it cannot read in place fall back to a copy."""
import ctypes

import pytest
import torch

import tda_b200
from tda_b200 import _lib

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _rand(shape, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(shape, generator=g).to(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("beta,norm", [(1.0, True), (0.5, False), (-0.5, True)])
def test_bshd_transposed_views_rect(D, beta, norm):
    B, S, H = 2, 200, 3
    q, k, v = (_rand((B, S, H, D), s).transpose(1, 2) for s in (1, 2, 3))  # (B, H, S, D) views
    assert not q.is_contiguous()
    out = tda_b200.rect_forward(q, k, v, beta, 2.0, norm)
    ref = tda_b200.rect_forward(q.contiguous(), k.contiguous(), v.contiguous(), beta, 2.0, norm)
    tda_b200.check_status()
    assert out.is_contiguous() and out.shape == (B, H, S, D)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("D", [64, 128])
def test_mixed_layouts_diff(D):
    """q1, k2 transposed views, q2 a head_dim slice of a wider tensor, k1 and
    v contiguous."""
    B, S, H = 1, 300, 4
    q1 = _rand((B, S, H, D), 11).transpose(1, 2)
    wide = _rand((B, H, S, 2 * D), 12)
    q2 = wide[..., D:]
    k1 = _rand((B, H, S, D), 13)
    k2 = _rand((B, S, H, D), 14).transpose(1, 2)
    v = _rand((B, H, S, D), 15)
    out = tda_b200.diff_forward(q1, q2, k1, k2, v, 1.0, 0.5, 2.0, True)
    ref = tda_b200.diff_forward(*(t.contiguous() for t in (q1, q2, k1, k2, v)), 1.0, 0.5, 2.0, True)
    tda_b200.check_status()
    assert torch.equal(out, ref)
    # and through the public autograd-aware function
    out2 = tda_b200.differential_threshold_rela_triton(q1, q2, k1, k2, v, torch.tensor(1.0), torch.tensor(0.5))
    assert torch.equal(out2, ref)


def test_strided_entry_through_c_abi():
    """The strided entry point called directly with (B, S, H, D) storage."""
    B, S, H, D = 2, 130, 2, 128
    xs = [_rand((B, S, H, D), 20 + i) for i in range(3)]
    lib = _lib.load()
    out = torch.empty((B, H, S, D), dtype=torch.bfloat16, device=DEV)
    ws_n = lib.tda_workspace_size(0, _lib.TDA_BF16, B * H, S, D, 1)
    ws = torch.empty(ws_n, dtype=torch.uint8, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = [S * H * D, D, H * D] * 3  # (batch, head, seq) element strides of (B, S, H, D) storage
    strides = (ctypes.c_int64 * 9)(*st)
    rc = lib.tda_rect_fwd_strided(*[x.data_ptr() for x in xs], ctypes.cast(strides, ctypes.c_void_p),
                                  out.data_ptr(), _lib.TDA_BF16, B, H, S, D, 1.0, 2.0, 1, ws.data_ptr(), ws_n,
                                  status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)
    ref = tda_b200.rect_forward(*(x.transpose(1, 2).contiguous() for x in xs), 1.0, 2.0, True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(out, ref)
    # strides that are not multiples of 8 elements are refused
    bad = (ctypes.c_int64 * 9)(*([S * H * D, D, H * D + 1] * 3))
    rc = lib.tda_rect_fwd_strided(*[x.data_ptr() for x in xs], ctypes.cast(bad, ctypes.c_void_p), out.data_ptr(),
                                  _lib.TDA_BF16, B, H, S, D, 1.0, 2.0, 1, ws.data_ptr(), ws_n, status.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.TDA_ERR_INVALID


def test_views_that_need_a_copy_still_work():
    """A transposed last dimension (stride(-1) != 1) cannot be read by TMA in
    place; the API copies it and the result is unchanged."""
    B, H, S, D = 1, 2, 128, 64
    base = _rand((B, H, D, S), 30)
    q = base.transpose(-1, -2)  # stride(-1) = S
    k, v = _rand((B, H, S, D), 31), _rand((B, H, S, D), 32)
    out = tda_b200.rect_forward(q, k, v, 1.0, 2.0, True)
    ref = tda_b200.rect_forward(q.contiguous(), k, v, 1.0, 2.0, True)
    assert torch.equal(out, ref)
