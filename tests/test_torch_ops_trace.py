"""The tda:: torch operators trace without a GPU: torch.compile(fullgraph=True)
over a module that calls the public functions runs end to end on meta
tensors (the operators' fake implementations give shapes and dtypes), forward
and backward, with no graph break."""
import torch

import tda_b200


class Block(torch.nn.Module):
    def forward(self, q1, q2, k1, k2, v, lam):
        a = tda_b200.differential_threshold_rela_triton(q1, q2, k1, k2, v, 1.0, lam, 2.0, True)
        b = tda_b200.threshold_rela_triton(q1, k1, v, 0.5, 2.0, True)
        return (a * 2.0 + b).float().sum()


def test_compile_fullgraph_traces_forward_and_backward_on_meta():
    torch._dynamo.reset()
    shape = (2, 4, 128, 64)
    xs = [torch.empty(shape, dtype=torch.bfloat16, device="meta", requires_grad=True) for _ in range(5)]
    lam = torch.empty((1, 4, 1, 1), device="meta", requires_grad=True)
    m = torch.compile(Block(), fullgraph=True, backend="aot_eager")
    loss = m(*xs, lam)
    assert loss.shape == () and loss.device.type == "meta"
    loss.backward()
    for x in xs:
        assert x.grad is not None and x.grad.shape == shape and x.grad.dtype == torch.bfloat16
    assert lam.grad is not None and lam.grad.shape == lam.shape


def test_operators_are_registered():
    for name in ("rect_fwd", "diff_fwd", "rect_bwd", "diff_bwd"):
        assert hasattr(torch.ops.tda, name)
