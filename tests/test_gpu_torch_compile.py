"""torch.compile(fullgraph=True) over a module that calls the public functions
(registered as the tda:: torch operators) matches eager execution bit for bit,
forward and backward; torch.library.opcheck validates the operators' schemas,
fake implementations and autograd registration on real CUDA inputs."""
import pytest
import torch

import tda_b200

pytestmark = pytest.mark.gpu

DEV = "cuda"


class Block(torch.nn.Module):
    """A differential attention layer followed by a rectified one, with
    ordinary torch ops around them."""

    def __init__(self, lam):
        super().__init__()
        self.lam = torch.nn.Parameter(lam)

    def forward(self, q1, q2, k1, k2, v):
        a = tda_b200.differential_threshold_rela_triton(q1, q2, k1, k2, v, 1.0, self.lam, 2.0, True)
        b = tda_b200.threshold_rela_triton(a, k1, v, 0.5, 2.0, True)
        return b * 0.5 + a


def _inputs(seed, shape):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return [torch.randn(shape, generator=g, device=DEV).to(torch.bfloat16).requires_grad_(True) for _ in range(5)]


def test_compile_fullgraph_matches_eager_bitwise():
    torch._dynamo.reset()
    shape = (2, 4, 256, 128)
    lam = torch.tensor([0.2, 0.5, 0.8, 1.0], device=DEV).view(1, 4, 1, 1)
    m = Block(lam.clone()).to(DEV)
    mc = torch.compile(Block(lam.clone()).to(DEV), fullgraph=True, backend="aot_eager")
    xe = _inputs(5, shape)
    xc = [x.detach().clone().requires_grad_(True) for x in xe]
    ye = m(*xe)
    yc = mc(*xc)
    assert torch.equal(ye, yc)
    g = torch.randn(ye.shape, device=DEV, generator=torch.Generator(device=DEV).manual_seed(6)).to(ye.dtype)
    ye.backward(g)
    yc.backward(g)
    for a, b in zip(xe, xc):
        assert torch.equal(a.grad, b.grad)
    assert torch.equal(m.lam.grad, mc._orig_mod.lam.grad)
    tda_b200.check_status()


def test_opcheck_operators():
    shape = (1, 2, 128, 64)
    xs = [x.detach() for x in _inputs(7, shape)]
    lam = torch.tensor(0.4, device=DEV)
    torch.library.opcheck(torch.ops.tda.rect_fwd.default, (xs[0], xs[2], xs[4], 1.0, 2.0, True))
    torch.library.opcheck(torch.ops.tda.diff_fwd.default, (*xs, 1.0, lam, 2.0, True))
    dout = torch.randn(shape, device=DEV).to(torch.bfloat16)
    torch.library.opcheck(torch.ops.tda.rect_bwd.default, (xs[0], xs[2], xs[4], dout, 1.0, 2.0, True))
    torch.library.opcheck(torch.ops.tda.diff_bwd.default, (*xs, dout, 1.0, lam, 2.0, True, True))
    tda_b200.check_status()
