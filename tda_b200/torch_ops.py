"""The tda_b200 forward and backward registered as torch operators.

    torch.ops.tda.rect_fwd(q, k, v, beta, relu_power, normalize) -> out
    torch.ops.tda.diff_fwd(q1, q2, k1, k2, v, beta, lambda_param, relu_power, normalize) -> out
    torch.ops.tda.rect_bwd(q, k, v, dout, beta, relu_power, normalize) -> (dq, dk, dv)
    torch.ops.tda.diff_bwd(q1, q2, k1, k2, v, dout, beta, lambda_param, relu_power, normalize,
                           need_dlam) -> (dq1, dq2, dk1, dk2, dv, dlambda)

The reference's entry points are a ``torch.autograd.Function``
(triton_threshold_attention.py:327) that torch can trace.  The CUDA library
here is called through ctypes, which a tracer cannot look into, so each call
is wrapped as an opaque operator with a fake (meta) implementation -- output
shapes and dtypes only -- and the forward ops carry their backward through
``register_autograd``.  ``torch.compile(fullgraph=True)`` therefore traces a
model that calls ``threshold_rela_triton`` / ``differential_threshold_rela_triton``
without a graph break, and its backward graph calls the backward ops.

Scalars: ``beta`` and ``relu_power`` are floats (the public functions read a
tensor ``beta`` once on the host, as the reference does at :352-353);
``lambda_param`` is a tensor (a float is turned into a 0-dim CPU tensor), read
on the device by the fused kernel when it lives there.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import ops


def _same_shapes(*ts):
    # reference :348
    assert all(t.shape == ts[0].shape for t in ts), "all inputs must have the same shape"


# ----------------------------------------------------------------- forward ops
@torch.library.custom_op("tda::rect_fwd", mutates_args=())
def rect_fwd(q: Tensor, k: Tensor, v: Tensor, beta: float, relu_power: float, normalize: bool) -> Tensor:
    """Threshold rectified attention forward (reference :472-486 -> :335-403)."""
    return ops.rect_forward(q, k, v, beta, relu_power, normalize)


@rect_fwd.register_fake
def _rect_fwd_fake(q, k, v, beta, relu_power, normalize):
    _same_shapes(q, k, v)
    return q.new_empty(q.shape)


@torch.library.custom_op("tda::diff_fwd", mutates_args=())
def diff_fwd(q1: Tensor, q2: Tensor, k1: Tensor, k2: Tensor, v: Tensor, beta: float, lambda_param: Tensor,
             relu_power: float, normalize: bool) -> Tensor:
    """Fused threshold differential attention forward (reference :489-519)."""
    return ops.diff_forward(q1, q2, k1, k2, v, beta, lambda_param, relu_power, normalize)


@diff_fwd.register_fake
def _diff_fwd_fake(q1, q2, k1, k2, v, beta, lambda_param, relu_power, normalize):
    _same_shapes(q1, q2, k1, k2, v)
    return q1.new_empty(q1.shape)


# ---------------------------------------------------------------- backward ops
@torch.library.custom_op("tda::rect_bwd", mutates_args=())
def rect_bwd(q: Tensor, k: Tensor, v: Tensor, dout: Tensor, beta: float, relu_power: float,
             normalize: bool) -> tuple[Tensor, Tensor, Tensor]:
    """(dq, dk, dv) of rect_fwd in the inputs' dtypes (reference :405-469)."""
    return ops.rect_grads(q, k, v, dout, beta, relu_power, normalize)


@rect_bwd.register_fake
def _rect_bwd_fake(q, k, v, dout, beta, relu_power, normalize):
    return q.new_empty(q.shape), k.new_empty(k.shape), v.new_empty(v.shape)


@torch.library.custom_op("tda::diff_bwd", mutates_args=())
def diff_bwd(q1: Tensor, q2: Tensor, k1: Tensor, k2: Tensor, v: Tensor, dout: Tensor, beta: float,
             lambda_param: Tensor, relu_power: float, normalize: bool,
             need_dlam: bool) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """(dq1, dq2, dk1, dk2, dv, dlambda) of diff_fwd; dlambda is zeros of
    lambda's shape when ``need_dlam`` is False."""
    g = ops.diff_grads(q1, q2, k1, k2, v, dout, beta, lambda_param, relu_power, normalize, need_dlam)
    dlam = g[5] if g[5] is not None else torch.zeros_like(lambda_param)
    return g[0], g[1], g[2], g[3], g[4], dlam


@diff_bwd.register_fake
def _diff_bwd_fake(q1, q2, k1, k2, v, dout, beta, lambda_param, relu_power, normalize, need_dlam):
    return (q1.new_empty(q1.shape), q2.new_empty(q2.shape), k1.new_empty(k1.shape), k2.new_empty(k2.shape),
            v.new_empty(v.shape), lambda_param.new_empty(lambda_param.shape))


# -------------------------------------------------------------------- autograd
def _rect_setup(ctx, inputs, output):
    q, k, v, beta, relu_power, normalize = inputs
    ctx.save_for_backward(q, k, v)
    ctx.args = (beta, relu_power, normalize)


def _rect_backward(ctx, dout):
    q, k, v = ctx.saved_tensors
    dq, dk, dv = torch.ops.tda.rect_bwd(q, k, v, dout, *ctx.args)
    return dq, dk, dv, None, None, None


rect_fwd.register_autograd(_rect_backward, setup_context=_rect_setup)


def _diff_setup(ctx, inputs, output):
    q1, q2, k1, k2, v, beta, lambda_param, relu_power, normalize = inputs
    ctx.save_for_backward(q1, q2, k1, k2, v, lambda_param)
    ctx.args = (beta, relu_power, normalize)


def _diff_backward(ctx, dout):
    q1, q2, k1, k2, v, lam = ctx.saved_tensors
    beta, relu_power, normalize = ctx.args
    need = bool(ctx.needs_input_grad[6])
    g = torch.ops.tda.diff_bwd(q1, q2, k1, k2, v, dout, beta, lam, relu_power, normalize, need)
    return g[0], g[1], g[2], g[3], g[4], None, (g[5] if need else None), None, None


diff_fwd.register_autograd(_diff_backward, setup_context=_diff_setup)
