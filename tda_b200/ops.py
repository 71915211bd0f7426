"""Host-side mirror of the reference TDA interface (snap-research/TDA,
``triton_threshold_attention.py``), backed by the tda_b200 C ABI.

Public functions keep the reference's names, argument meaning and error
behaviour:

* ``threshold_rela_triton(q, k, v, beta, relu_power=2.0, normalize=False)``
  -- reference :472-486.  ``normalize`` is an added trailing keyword; its
  default (False) is the reference's behaviour, True equals the reference
  called on F.normalize(q), F.normalize(k).
* ``differential_threshold_rela_triton(q1, q2, k1, k2, v, beta, lambda_param,
  relu_power=2.0, normalize=True)`` -- reference :489-519, computed in ONE
  fused pass over the keys (one launch instead of two forward kernels plus
  the torch normalize / clamp / combine ops).
* ``ThresholdRelaFunction`` -- reference :327-469, forward and backward
  (``rect_backward``: the reference's dQ / dK / dV kernels, :118-324; bf16 at
  head_dim 64/128 on the tcgen05 tensor cores, fp32 and head_dim 16/32 in
  exact fp32 on CUDA cores).

Forward data path: CUDA tensors only.  bf16 with head_dim 64/128 runs the
tcgen05 tensor-core kernel, and so does fp16 with head_dim 64/128 when
normalized (fp16 operands; P bounded); fp32 with head_dim 64/128 runs the tcgen05 kind::tf32
kernel with three TF32 products per fp32 product (fp32 accuracy); fp32 at
other head dims runs the exact-fp32 CUDA-core kernel; other dtypes / head dims
are widened to fp32 on the device.  There is no CPU fallback: CPU tensors
raise, and a missing CUDA library raises.
"""
from __future__ import annotations

import os

import torch

from . import _lib

_STATUS: dict[int, torch.Tensor] = {}
_SYNC_CHECK = os.environ.get("TDA_B200_SYNC_CHECK", "0") not in ("", "0")


def _status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def check_status(device=None, reset: bool = True) -> None:
    """Synchronise ``device`` and raise if any tda_b200 kernel on it reported a
    bounded wait that gave up (its output is then invalid).  Clears the word
    when ``reset``."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    word = _status_word(dev)
    code = int(word.item())
    if code != 0:
        if reset:
            word.zero_()
        raise _lib.TdaError(f"tda_b200 kernel aborted after a wait timeout (status 0x{code:x})")


def _scalar(x) -> float:
    # reference :352-353: Tensor -> .item(), else float()
    return float(x.item()) if isinstance(x, torch.Tensor) else float(x)


def _fp16_ok(normalize: bool, beta: float, p: float, S: int, D: int) -> bool:
    """fp16 operands on the tensor cores need P = relu(z)^p bounded (its fp16
    hi + lo split): normalize, p > 0 and (1 + max(0, -beta) sqrt(2 ln S / D))^p
    <= 16384 -- the rule the C library applies (tda_b200.h)."""
    import math
    if not normalize or not p > 0.0:
        return False
    tau_max = -beta * math.sqrt(2.0 * math.log(S) / D) if beta < 0.0 else 0.0
    try:
        return (1.0 + tau_max) ** p <= 16384.0
    except OverflowError:
        return False


def _plan(tensors, what: str, normalize: bool = False, beta: float = 0.0, p: float = 2.0):
    """Validate device / shape and pick the kernel path.  Returns
    (kind, compute_tensors, orig_dtype): bf16 (head_dim 64 / 128) and fp16
    (head_dim 64 / 128, normalized, P bounded) run on the tensor cores in
    their own type; everything else is widened to fp32."""
    t0 = tensors[0]
    for t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{what}: expected torch.Tensor inputs")
    if t0.dim() != 4:
        raise ValueError(f"{what}: expected (batch, num_heads, seq_len, head_dim) tensors, got {tuple(t0.shape)}")
    if not t0.is_cuda:
        raise RuntimeError(f"{what}: tda_b200 runs on CUDA tensors only (got device {t0.device}); "
                           "there is no CPU fallback")
    for t in tensors:
        if t.device != t0.device:
            raise RuntimeError(f"{what}: all inputs must be on one device")
    orig = t0.dtype
    common = tensors[0].dtype
    for t in tensors[1:]:
        common = torch.promote_types(common, t.dtype)
    if not common.is_floating_point:
        raise TypeError(f"{what}: floating point inputs required, got {common}")
    D = t0.shape[-1]
    if D < 16 or D > 256 or (D & (D - 1)) != 0:
        raise ValueError(f"{what}: head_dim must be a power of two in [16, 256], got {D}")
    if common == torch.bfloat16 and D in (64, 128):
        kind, cdt = _lib.TDA_BF16, torch.bfloat16
    elif common == torch.float16 and D in (64, 128) and _fp16_ok(normalize, beta, p, t0.shape[2], D):
        kind, cdt = _lib.TDA_F16, torch.float16
    else:
        kind, cdt = _lib.TDA_F32, torch.float32
    comp = [t.to(cdt).contiguous() for t in tensors]
    return kind, comp, orig


_KIND_OF = {torch.float32: _lib.TDA_F32, torch.bfloat16: _lib.TDA_BF16, torch.float16: _lib.TDA_F16}


def _raw_dtype(kind: int, out_dtype) -> torch.dtype:
    """Element type the kernel writes: the compute type, or fp32 when asked
    for (the accumulator of a bf16 / fp16 computation)."""
    if kind == _lib.TDA_F32 or out_dtype == torch.float32:
        return torch.float32
    return torch.float16 if kind == _lib.TDA_F16 else torch.bfloat16


def _finish(out: torch.Tensor, orig: torch.dtype, out_dtype) -> torch.Tensor:
    want = orig if out_dtype is None else out_dtype
    if out.dtype != want:
        out = out.to(want)
    if _SYNC_CHECK:
        check_status(out.device)
    return out


def _strided_eligible(ts) -> bool:
    """bf16 CUDA views the tensor-core kernel can read in place: same device,
    contiguous last dimension, head_dim 64 / 128, element strides of the first
    three dimensions positive multiples of 8, 16-byte aligned data."""
    t0 = ts[0]
    if t0.dim() != 4 or t0.shape[-1] not in (64, 128) or not t0.is_cuda:
        return False
    for t in ts:
        if t.dtype != torch.bfloat16 or t.device != t0.device or t.stride(-1) != 1 or t.data_ptr() % 16:
            return False
        if any(x <= 0 or x % 8 for x in t.stride()[:3]):
            return False
    return not all(t.is_contiguous() for t in ts)


def _device_lambda(lam, B: int, H: int, device):
    """A tensor lambda that varies at most over (batch, head), as an fp32
    device tensor and its element strides (batch, head), 0 for a broadcast
    dimension.  None for a host scalar (a float or a one-element CPU tensor,
    read once like the reference reads its scalars) and for a lambda that
    varies along the sequence or head_dim axes (or has more than 4 dims)."""
    if not isinstance(lam, torch.Tensor) or lam.dim() > 4:
        return None
    if not lam.is_cuda and lam.numel() == 1:
        return None
    l4 = lam[(None,) * (4 - lam.dim())]
    if l4.shape[2] != 1 or l4.shape[3] != 1 or l4.shape[0] not in (1, B) or l4.shape[1] not in (1, H):
        return None
    if l4.device != device or l4.dtype != torch.float32:
        l4 = l4.to(device=device, dtype=torch.float32)
    sb = l4.stride(0) if l4.shape[0] != 1 else 0
    sh = l4.stride(1) if l4.shape[1] != 1 else 0
    return l4, sb, sh


def _diff_lambda_call(ts, strided, kind, out, lam_dev, beta_v, p_v, normalize):
    """tda_diff_fwd_lambda: the fused differential forward with lambda read on
    the device per (batch, head)."""
    import ctypes
    B, H, S, D = ts[0].shape
    lib = _lib.load()
    lt, sb, sh = lam_dev
    ws_n = lib.tda_workspace_size(1, kind, B * H, S, D, int(normalize))
    ws = torch.empty(ws_n, dtype=torch.uint8, device=out.device) if ws_n else None
    strides = None
    if strided:
        strides = (ctypes.c_int64 * 15)(*[x for t in ts for x in t.stride()[:3]])
    out_kind = _KIND_OF[out.dtype]
    stream = torch.cuda.current_stream(out.device).cuda_stream
    with torch.cuda.device(out.device):
        rc = lib.tda_diff_fwd_lambda(*[t.data_ptr() for t in ts],
                                     ctypes.cast(strides, ctypes.c_void_p) if strides is not None else None,
                                     out.data_ptr(), kind, out_kind, B, H, S, D, beta_v, lt.data_ptr(), sb, sh, p_v,
                                     int(normalize), ws.data_ptr() if ws is not None else None, ws_n,
                                     _status_word(out.device).data_ptr(), stream)
    _lib.check(rc)
    return out


def _strided_call(entry, ts, out_dtype, extra, normalize, differential):
    import ctypes
    B, H, S, D = ts[0].shape
    raw_dt = torch.float32 if out_dtype == torch.float32 else torch.bfloat16
    out = torch.empty((B, H, S, D), dtype=raw_dt, device=ts[0].device)
    if out.numel() == 0:
        return out
    lib = _lib.load()
    ws_n = lib.tda_workspace_size(int(differential), _lib.TDA_BF16, B * H, S, D, int(normalize))
    ws = torch.empty(ws_n, dtype=torch.uint8, device=out.device) if ws_n else None
    strides = (ctypes.c_int64 * (3 * len(ts)))(*[x for t in ts for x in t.stride()[:3]])
    out_kind = _KIND_OF[raw_dt]
    stream = torch.cuda.current_stream(out.device).cuda_stream
    with torch.cuda.device(out.device):
        rc = getattr(lib, entry)(*[t.data_ptr() for t in ts], ctypes.cast(strides, ctypes.c_void_p),
                                 out.data_ptr(), out_kind, B, H, S, D, *extra, int(normalize),
                                 ws.data_ptr() if ws is not None else None, ws_n,
                                 _status_word(out.device).data_ptr(), stream)
    _lib.check(rc)
    return out


def rect_forward(q, k, v, beta, relu_power=2.0, normalize: bool = False, out_dtype=None) -> torch.Tensor:
    """Threshold rectified attention forward (no autograd).  ``out_dtype``
    (default: q's dtype) may be torch.float32 on the bf16 path to receive the
    kernel's fp32 accumulator."""
    # reference :348
    assert q.shape == k.shape == v.shape
    beta_v = _scalar(beta)
    p_v = _scalar(relu_power)
    if _strided_eligible([q, k, v]):
        # strided views (e.g. (B, S, H, D) transposed) are read in place
        out = _strided_call("tda_rect_fwd_strided", [q, k, v], out_dtype, (beta_v, p_v), normalize, False)
        return _finish(out, q.dtype, out_dtype)
    kind, (qc, kc, vc), orig = _plan([q, k, v], "threshold_rela_triton", normalize, beta_v, p_v)
    B, H, S, D = qc.shape
    raw_dt = _raw_dtype(kind, out_dtype)
    out = torch.empty((B, H, S, D), dtype=raw_dt, device=qc.device)
    if out.numel() == 0:
        return _finish(out, orig, out_dtype)
    lib = _lib.load()
    ws_n = lib.tda_workspace_size(0, kind, B * H, S, D, int(normalize))
    ws = torch.empty(ws_n, dtype=torch.uint8, device=qc.device) if ws_n else None
    stream = torch.cuda.current_stream(qc.device).cuda_stream
    out_kind = _KIND_OF[raw_dt]
    with torch.cuda.device(qc.device):
        rc = lib.tda_rect_fwd(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), kind, out_kind,
                              B * H, S, D, beta_v, p_v, int(normalize),
                              ws.data_ptr() if ws is not None else None, ws_n,
                              _status_word(qc.device).data_ptr(), stream)
    _lib.check(rc)
    return _finish(out, orig, out_dtype)


def diff_forward(q1, q2, k1, k2, v, beta, lambda_param, relu_power=2.0, normalize: bool = True,
                 out_dtype=None) -> torch.Tensor:
    """Threshold differential attention forward (no autograd), fused.

    lambda_param: a float, or a tensor broadcastable against the output.  A
    host scalar (float, one-element CPU tensor) is read once; a CUDA tensor
    that varies at most over (batch, head) -- a scalar, per head or per
    (batch, head) -- is read by the kernel itself (no host synchronisation,
    one fused pass); a lambda that also varies along the sequence or head_dim
    axes runs the two branches separately and combines them as the reference
    does (:516-517)."""
    assert q1.shape == q2.shape == k1.shape == k2.shape == v.shape
    beta_v = _scalar(beta)
    p_v = _scalar(relu_power)
    lam_dev = None
    if isinstance(lambda_param, torch.Tensor) and q1.dim() == 4 and q1.is_cuda:
        lam_dev = _device_lambda(lambda_param, q1.shape[0], q1.shape[1], q1.device)
        if lam_dev is None and lambda_param.numel() != 1:
            # lambda varying along the sequence / head_dim axes: the
            # reference's combine out1 - clamp(lambda) * out2 on two passes
            o1 = rect_forward(q1, k1, v, beta_v, p_v, normalize, out_dtype=torch.float32)
            o2 = rect_forward(q2, k2, v, beta_v, p_v, normalize, out_dtype=torch.float32)
            lam = torch.clamp(lambda_param.to(device=o1.device, dtype=torch.float32), min=0.0, max=1.0)
            return _finish(o1 - lam * o2, q1.dtype, out_dtype)
    if _strided_eligible([q1, q2, k1, k2, v]):
        if lam_dev is not None:
            B, H, S, D = q1.shape
            out = torch.empty((B, H, S, D), dtype=torch.float32 if out_dtype == torch.float32 else torch.bfloat16,
                              device=q1.device)
            out = _diff_lambda_call([q1, q2, k1, k2, v], True, _lib.TDA_BF16, out, lam_dev, beta_v, p_v, normalize)
            return _finish(out, q1.dtype, out_dtype)
        out = _strided_call("tda_diff_fwd_strided", [q1, q2, k1, k2, v], out_dtype,
                            (beta_v, _scalar(lambda_param), p_v), normalize, True)
        return _finish(out, q1.dtype, out_dtype)
    kind, (a, b, c, d, e), orig = _plan([q1, q2, k1, k2, v], "differential_threshold_rela_triton", normalize, beta_v,
                                        p_v)
    B, H, S, D = a.shape
    raw_dt = _raw_dtype(kind, out_dtype)
    out = torch.empty((B, H, S, D), dtype=raw_dt, device=a.device)
    if out.numel() == 0:
        return _finish(out, orig, out_dtype)
    if lam_dev is not None:
        out = _diff_lambda_call([a, b, c, d, e], False, kind, out, lam_dev, beta_v, p_v, normalize)
        return _finish(out, orig, out_dtype)
    lam_v = _scalar(lambda_param)
    lib = _lib.load()
    ws_n = lib.tda_workspace_size(1, kind, B * H, S, D, int(normalize))
    ws = torch.empty(ws_n, dtype=torch.uint8, device=a.device) if ws_n else None
    stream = torch.cuda.current_stream(a.device).cuda_stream
    out_kind = _KIND_OF[raw_dt]
    with torch.cuda.device(a.device):
        rc = lib.tda_diff_fwd(a.data_ptr(), b.data_ptr(), c.data_ptr(), d.data_ptr(), e.data_ptr(), out.data_ptr(),
                              kind, out_kind, B * H, S, D, beta_v, lam_v, p_v, int(normalize),
                              ws.data_ptr() if ws is not None else None, ws_n,
                              _status_word(a.device).data_ptr(), stream)
    _lib.check(rc)
    return _finish(out, orig, out_dtype)


def rect_backward(q, k, v, dout, beta, relu_power=2.0, normalize: bool = False, dout_scale: float = 1.0,
                  dv: torch.Tensor | None = None):
    """Gradients (dq, dk, dv), fp32, of ``rect_forward(q, k, v, beta, p,
    normalize)`` for the upstream gradient ``dout_scale * dout``, as the
    reference's backward computes them (:405-469, kernels :118-324; masked
    entries included in dQ / dK, which matters for beta < 0).  When ``dv`` (an
    fp32 tensor of v's shape) is given, the value gradient is added into it."""
    assert q.shape == k.shape == v.shape == dout.shape
    beta_v = _scalar(beta)
    p_v = _scalar(relu_power)
    for t in (q, k, v, dout):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError("threshold attention backward: tda_b200 runs on CUDA tensors only; "
                               "there is no CPU fallback")
    B, H, S, D = q.shape
    all_bf16 = all(t.dtype == torch.bfloat16 for t in (q, k, v, dout))
    kind, cdt = (_lib.TDA_BF16, torch.bfloat16) if all_bf16 else (_lib.TDA_F32, torch.float32)
    qc, kc, vc, gc = (t.to(cdt).contiguous() for t in (q, k, v, dout))
    dq = torch.empty((B, H, S, D), dtype=torch.float32, device=qc.device)
    dk = torch.empty_like(dq)
    accumulate = dv is not None
    if dv is None:
        dv = torch.empty_like(dq)
    elif dv.dtype != torch.float32 or not dv.is_contiguous() or dv.shape != dq.shape:
        raise ValueError("dv must be a contiguous fp32 tensor of v's shape")
    if dq.numel() == 0:
        return dq, dk, dv
    lib = _lib.load()
    ws_n = lib.tda_bwd_workspace_size(kind, B * H, S, D, int(normalize))
    ws = torch.empty(ws_n, dtype=torch.uint8, device=qc.device) if ws_n else None
    stream = torch.cuda.current_stream(qc.device).cuda_stream
    with torch.cuda.device(qc.device):
        rc = lib.tda_rect_bwd(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), gc.data_ptr(), kind, dq.data_ptr(),
                              dk.data_ptr(), dv.data_ptr(), B * H, S, D, beta_v, p_v, int(normalize),
                              float(dout_scale), int(accumulate), ws.data_ptr() if ws is not None else None, ws_n,
                              _status_word(qc.device).data_ptr(), stream)
    _lib.check(rc)
    if _SYNC_CHECK:
        check_status(qc.device)
    return dq, dk, dv


def rect_grads(q, k, v, dout, beta, relu_power, normalize):
    """(dq, dk, dv) of ``rect_forward(q, k, v, beta, relu_power, normalize)``
    for the upstream gradient ``dout``, in the inputs' dtypes (reference
    ThresholdRelaFunction.backward :405-469)."""
    dq, dk, dv = rect_backward(q, k, v, dout, beta, relu_power, normalize)
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


def diff_grads(q1, q2, k1, k2, v, dout, beta, lambda_param, relu_power, normalize, need_dlam: bool):
    """(dq1, dq2, dk1, dk2, dv, dlambda) of the differential form for the
    upstream gradient ``dout``: each branch through the branch backward (branch
    2 with -clamp(lambda) * dout, dv summed), and d lambda = -sum(out2 * dout)
    where torch.clamp passes the gradient (0 <= lambda <= 1), as torch
    autograd gives it around the reference (:512-517).  ``lambda_param`` is a
    float or a tensor; dlambda (lambda's shape and dtype) only when
    ``need_dlam`` and lambda is a tensor, else None."""
    lam_t = lambda_param if isinstance(lambda_param, torch.Tensor) else None
    dq1, dk1, dv = rect_backward(q1, k1, v, dout, beta, relu_power, normalize)
    if lam_t is None or (lam_t.numel() == 1 and not lam_t.is_cuda):
        lam = float(lambda_param) if lam_t is None else _scalar(lam_t)
        lamc = min(max(lam, 0.0), 1.0)
        dq2, dk2, dv = rect_backward(q2, k2, v, dout, beta, relu_power, normalize, dout_scale=-lamc, dv=dv)
    else:
        # tensor lambda (on the device, or broadcast): the second branch
        # sees -clamp(lambda) * dout, formed without reading lambda on the host
        lamc = torch.clamp(lam_t.to(device=dout.device, dtype=torch.float32), min=0.0, max=1.0)
        d2 = (-lamc * dout.float()).contiguous()
        dq2, dk2, dv = rect_backward(q2, k2, v, d2, beta, relu_power, normalize, dv=dv)
    dlam = None
    if lam_t is not None and need_dlam:
        o2 = rect_forward(q2, k2, v, beta, relu_power, normalize, out_dtype=torch.float32)
        g = -(o2 * dout.float())
        lam32 = lam_t.to(device=dout.device, dtype=torch.float32)
        inside = ((lam32 >= 0.0) & (lam32 <= 1.0)).to(torch.float32)
        dlam = (g.sum() * inside if lam_t.numel() == 1 else g.sum_to_size(lam_t.shape) * inside)
        dlam = dlam.reshape(lam_t.shape).to(device=lam_t.device, dtype=lam_t.dtype)
    return (dq1.to(q1.dtype), dq2.to(q2.dtype), dk1.to(k1.dtype), dk2.to(k2.dtype), dv.to(v.dtype), dlam)


class ThresholdRelaFunction(torch.autograd.Function):
    """Threshold Rectified Attention (reference :327-469).

    forward(q, k, v, beta, relu_power[, normalize]) -> out; backward returns
    dq, dk, dv in the inputs' dtypes (beta and relu_power get no gradient, as
    in the reference, :469)."""

    @staticmethod
    def forward(ctx, q, k, v, beta, relu_power, normalize=False):
        out = rect_forward(q, k, v, beta, relu_power, normalize)
        ctx.save_for_backward(q, k, v)
        ctx.beta = _scalar(beta)
        ctx.relu_power = _scalar(relu_power)
        ctx.normalize = bool(normalize)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v = ctx.saved_tensors
        dq, dk, dv = rect_grads(q, k, v, dout, ctx.beta, ctx.relu_power, ctx.normalize)
        return dq, dk, dv, None, None, None


class DifferentialThresholdRelaFunction(torch.autograd.Function):
    """Fused threshold differential attention as an autograd Function
    (gradients: ``diff_grads``)."""

    @staticmethod
    def forward(ctx, q1, q2, k1, k2, v, beta, lambda_param, relu_power, normalize):
        out = diff_forward(q1, q2, k1, k2, v, beta, lambda_param, relu_power, normalize)
        lam_t = lambda_param if isinstance(lambda_param, torch.Tensor) else None
        ctx.save_for_backward(q1, q2, k1, k2, v, lam_t)
        ctx.lam_float = None if lam_t is not None else float(lambda_param)
        ctx.beta = _scalar(beta)
        ctx.relu_power = _scalar(relu_power)
        ctx.normalize = bool(normalize)
        return out

    @staticmethod
    def backward(ctx, dout):
        q1, q2, k1, k2, v, lam_t = ctx.saved_tensors
        lam = ctx.lam_float if lam_t is None else lam_t
        g = diff_grads(q1, q2, k1, k2, v, dout, ctx.beta, lam, ctx.relu_power, ctx.normalize,
                       ctx.needs_input_grad[6])
        return g[0], g[1], g[2], g[3], g[4], None, g[5], None, None


def threshold_rela_triton(q, k, v, beta, relu_power=2.0, normalize=False):
    """Threshold Rectified Attention: out = ReLU(Q K^T - tau)^p V, causal.

    q, k, v: (batch, num_heads, seq_len, head_dim); beta: scalar tensor or
    float; relu_power: scalar (default 2.0); normalize: L2-normalize q and k
    first (default False, the reference's behaviour).  Returns a tensor of
    q's shape and dtype.  Runs as the torch operator ``tda::rect_fwd``
    (differentiable, traceable by torch.compile)."""
    return torch.ops.tda.rect_fwd(q, k, v, _scalar(beta), _scalar(relu_power), bool(normalize))


def differential_threshold_rela_triton(q1, q2, k1, k2, v, beta, lambda_param, relu_power=2.0, normalize=True):
    """Threshold Differential Attention:
    out = TRA(q1, k1, v) - clamp(lambda, 0, 1) * TRA(q2, k2, v), with q/k
    L2-normalized when ``normalize`` (default True).  lambda_param: a tensor
    broadcastable against the output (a float is accepted too).  Returns
    q1's shape and dtype.  Runs as the torch operator ``tda::diff_fwd``
    (differentiable, traceable by torch.compile)."""
    lam = lambda_param if isinstance(lambda_param, torch.Tensor) else torch.tensor(float(lambda_param))
    return torch.ops.tda.diff_fwd(q1, q2, k1, k2, v, _scalar(beta), lam, _scalar(relu_power), bool(normalize))
