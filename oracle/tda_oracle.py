"""CPU restatement of the TDA forward and backward passes -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA path, never the thing measured or
shipped.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` may import it.  The product path in ``tda_b200`` never calls it
and fails loudly when its CUDA library is missing.

It restates, in numpy, the arithmetic of the reference ``triton_threshold_attention.py``
(snap-research/TDA):

* ``_threshold_rela_fwd_kernel``  (triton_threshold_attention.py:19-115)
    - tau(i) = beta * sqrt(2 * log(i + 1) / D), computed in fp32   (:59-63)
    - scores  s_ij = q_i . k_j  over every key j < S                (:66-75)
    - causal mask: s_ij = 0 (not -inf) for j > i                    (:77-80)
    - x_ij = relu(s_ij - tau_i)                                     (:82-87)
    - P_ij = x^2 if p == 2, x if p == 1,
             exp(p * log(x + 1e-10)) where x > 0 otherwise          (:89-101)
    - out_i = sum_j P_ij v_j                                        (:103-109)
* ``differential_threshold_rela_triton``  (triton_threshold_attention.py:489-519)
    - optional F.normalize(p=2, dim=-1, eps=1e-12) of q1, k1, q2, k2 (:505-509)
    - out = rect(q1, k1, v) - clamp(lambda, 0, 1) * rect(q2, k2, v) (:512-517)
* the backward kernels ``_threshold_rela_bwd_kernel_dq`` / ``_dkv``
  (triton_threshold_attention.py:118-324) and ``ThresholdRelaFunction.backward``
  (:405-469), plus the gradients torch autograd adds around them in the
  differential form (F.normalize, clamp(lambda), the combine)
* ``threshold_rela_triton``  (triton_threshold_attention.py:472-486) has no
  ``normalize`` argument in the reference; ``normalize=True`` here means the
  reference called on F.normalize(q), F.normalize(k), exactly as each branch of
  the differential form does.

Parity is pinned against outputs of the reference itself, run on CPU under
``TRITON_INTERPRET=1`` (see ``tests/golden/make_golden.py`` and
``tests/test_oracle_golden.py``).

The default arithmetic is float64 (the accuracy oracle).  ``dtype=np.float32``
gives the same formula in fp32, which is what the CPU baseline times.
"""
from __future__ import annotations

import numpy as np

NORM_EPS = 1e-12  # torch.nn.functional.normalize default eps (triton_threshold_attention.py:506)
POW_EPS = 1e-10   # bias inside log for the general power (triton_threshold_attention.py:99)


def tau_vector(seq_len: int, head_dim: int, beta: float) -> np.ndarray:
    """Per-row threshold tau(i) = beta*sqrt(2*log(i+1)/D) in fp32, as at
    triton_threshold_attention.py:62-63 (row index promoted to fp32 first)."""
    rows = np.arange(seq_len, dtype=np.float32) + np.float32(1.0)
    return (np.float32(beta) * np.sqrt((np.float32(2.0) * np.log(rows)) / np.float32(head_dim))).astype(np.float32)


def l2_normalize(x: np.ndarray, dtype=np.float64) -> np.ndarray:
    """x / max(||x||_2, eps) along the last axis (torch F.normalize semantics)."""
    x = np.asarray(x, dtype=dtype)
    n = np.sqrt(np.sum(x * x, axis=-1, keepdims=True))
    return x / np.maximum(n, dtype(NORM_EPS))


def relu_power(x: np.ndarray, p: float) -> np.ndarray:
    """The power branch of triton_threshold_attention.py:89-101 applied to x >= 0."""
    if p == 2.0:
        return x * x
    if p == 1.0:
        return x
    with np.errstate(divide="ignore"):
        y = np.exp(x.dtype.type(p) * np.log(x + x.dtype.type(POW_EPS)))
    return np.where(x > 0, y, x.dtype.type(0))


def _as_bhsd(x) -> np.ndarray:
    x = np.asarray(x)
    if x.ndim != 4:
        raise ValueError("expected a (batch, heads, seq_len, head_dim) array")
    return x


def rect_fwd(q, k, v, beta, relu_power_: float = 2.0, normalize: bool = False,
             dtype=np.float64, rows=None, bh=None, row_chunk: int = 512) -> np.ndarray:
    """Threshold rectified attention forward (triton_threshold_attention.py:19-115).

    q, k, v: (B, H, S, D) arrays of any float type (bf16 inputs should be passed
    already widened to float32).  Returns (B, H, S, D) in ``dtype``.

    ``bh`` (iterable of flat batch*head indices) and ``rows`` (iterable of query
    rows) restrict the computation to a sample; other entries are left as NaN.
    """
    q, k, v = _as_bhsd(q), _as_bhsd(k), _as_bhsd(v)
    if not (q.shape == k.shape == v.shape):
        raise AssertionError("q, k, v must have the same shape")
    B, H, S, D = q.shape
    beta = float(beta)
    p = float(relu_power_)
    tau = tau_vector(S, D, beta).astype(dtype)
    qf = q.reshape(B * H, S, D)
    kf = k.reshape(B * H, S, D)
    vf = v.reshape(B * H, S, D)
    out = np.full((B * H, S, D), np.nan, dtype=dtype)
    bh_list = range(B * H) if bh is None else list(bh)
    row_list = np.arange(S) if rows is None else np.asarray(sorted(set(int(r) for r in rows)))
    zero = dtype(0)
    for b in bh_list:
        kb = kf[b].astype(dtype)
        qb = qf[b].astype(dtype)
        if normalize:
            kb = l2_normalize(kb, dtype)
            qb = l2_normalize(qb, dtype)
        vb = vf[b].astype(dtype)
        for c0 in range(0, len(row_list), row_chunk):
            r = row_list[c0:c0 + row_chunk]
            # with beta >= 0 the masked entries give relu(0 - tau) = 0, so keys
            # beyond the last row of the chunk can be dropped without changing
            # the result; with beta < 0 every key contributes (mask-to-zero).
            nk = S if beta < 0 else int(r.max()) + 1
            s = qb[r] @ kb[:nk].T
            mask = np.arange(nk)[None, :] <= r[:, None]
            s = np.where(mask, s, zero)
            x = np.maximum(s - tau[r][:, None], zero)
            out[b, r] = relu_power(x, p) @ vb[:nk]
    return out.reshape(B, H, S, D)


def diff_fwd(q1, q2, k1, k2, v, beta, lambda_param, relu_power_: float = 2.0,
             normalize: bool = True, dtype=np.float64, rows=None, bh=None) -> np.ndarray:
    """Threshold differential attention (triton_threshold_attention.py:489-519):
    rect(q1,k1,v) - clamp(lambda,0,1) * rect(q2,k2,v), both branches normalized
    when ``normalize``."""
    lam = min(max(float(lambda_param), 0.0), 1.0)
    o1 = rect_fwd(q1, k1, v, beta, relu_power_, normalize, dtype, rows, bh)
    o2 = rect_fwd(q2, k2, v, beta, relu_power_, normalize, dtype, rows, bh)
    return o1 - dtype(lam) * o2


def relu_power_grad(z: np.ndarray, p: float) -> np.ndarray:
    """d relu(z)^p / dz as the reference's backward kernels form it
    (triton_threshold_attention.py:195-206 and :294-304): 2 relu(z) for p == 2,
    1{z > 0} for p == 1, else p * exp((p - 1) * log(relu(z) + 1e-10)) where
    relu(z) > 0."""
    x = np.maximum(z, z.dtype.type(0))
    if p == 2.0:
        return z.dtype.type(2) * x
    if p == 1.0:
        return np.where(z > 0, z.dtype.type(1), z.dtype.type(0))
    with np.errstate(divide="ignore"):
        y = z.dtype.type(p) * np.exp(z.dtype.type(p - 1.0) * np.log(x + z.dtype.type(POW_EPS)))
    return np.where(x > 0, y, z.dtype.type(0))


def rect_bwd_core(q, k, v, dout, beta, relu_power_: float = 2.0, dtype=np.float64,
                  row_chunk: int = 512):
    """Gradients of the rectified forward w.r.t. its (already normalized) q, k
    and v, formed as the reference's two backward kernels form them
    (triton_threshold_attention.py:118-224 for dQ, :227-324 for dK / dV):

      s_ij  = q_i . k_j, set to 0 for j > i          (recomputed, :186-190, :282-286)
      z_ij  = s_ij - tau_i
      dP_ij = dout_i . v_j                             (:211, :312)
      dA_ij = dP_ij * relu_power_grad(z_ij)            (:214, :313)
      dq_i  = sum_j dA_ij k_j     over every key j     (:219)
      dk_j  = sum_i dA_ij q_i     over every query i   (:317)
      dv_j  = sum_i relu(z_ij)^p dout_i                (:307)

    The mask zeroes s_ij but dA_ij is not masked, so with beta < 0 (tau < 0,
    z_ij = -tau_i > 0 on masked entries) the reference's dq and dk take
    contributions from keys after the query row; they are kept here.  With
    beta >= 0 those entries have zero gradient.  Returns (dq, dk, dv) shaped
    like q, in ``dtype``.
    """
    q, k, v, dout = _as_bhsd(q), _as_bhsd(k), _as_bhsd(v), _as_bhsd(dout)
    B, H, S, D = q.shape
    p = float(relu_power_)
    tau = tau_vector(S, D, float(beta)).astype(dtype)
    qf, kf, vf, gf = (x.reshape(B * H, S, D).astype(dtype) for x in (q, k, v, dout))
    dq = np.zeros((B * H, S, D), dtype=dtype)
    dk = np.zeros_like(dq)
    dv = np.zeros_like(dq)
    zero = dtype(0)
    keys = np.arange(S)
    for b in range(B * H):
        for c0 in range(0, S, row_chunk):
            r = np.arange(c0, min(S, c0 + row_chunk))
            s = qf[b, r] @ kf[b].T
            s = np.where(keys[None, :] <= r[:, None], s, zero)
            z = s - tau[r][:, None]
            x = np.maximum(z, zero)
            P = relu_power(x, p)
            dA = (gf[b, r] @ vf[b].T) * relu_power_grad(z, p)
            dq[b, r] = dA @ kf[b]
            dk[b] += dA.T @ qf[b, r]
            dv[b] += P.T @ gf[b, r]
    return tuple(x.reshape(B, H, S, D) for x in (dq, dk, dv))


def l2_normalize_bwd(x, g, dtype=np.float64) -> np.ndarray:
    """Gradient through y = x / max(||x||, eps) (torch F.normalize): for
    ||x|| > eps, (g - y (y . g)) / ||x||; otherwise g / eps."""
    x = np.asarray(x, dtype=dtype)
    g = np.asarray(g, dtype=dtype)
    n = np.sqrt(np.sum(x * x, axis=-1, keepdims=True))
    big = n > dtype(NORM_EPS)
    nn = np.where(big, n, dtype(1))
    y = x / nn
    gx = (g - y * np.sum(y * g, axis=-1, keepdims=True)) / nn
    return np.where(big, gx, g / dtype(NORM_EPS))


def rect_bwd(q, k, v, dout, beta, relu_power_: float = 2.0, normalize: bool = False,
             dtype=np.float64):
    """Gradients of ``rect_fwd(q, k, v, beta, p, normalize)`` w.r.t. q, k, v:
    the reference's backward kernels on F.normalize'd q, k when ``normalize``,
    chained through F.normalize (as torch autograd does around the reference
    op, triton_threshold_attention.py:505-512)."""
    qn = l2_normalize(q, dtype) if normalize else np.asarray(q, dtype=dtype)
    kn = l2_normalize(k, dtype) if normalize else np.asarray(k, dtype=dtype)
    dq, dk, dv = rect_bwd_core(qn, kn, v, dout, beta, relu_power_, dtype)
    if normalize:
        dq = l2_normalize_bwd(q, dq, dtype)
        dk = l2_normalize_bwd(k, dk, dtype)
    return dq, dk, dv


def diff_bwd(q1, q2, k1, k2, v, dout, beta, lambda_param, relu_power_: float = 2.0,
             normalize: bool = True, dtype=np.float64):
    """Gradients of ``diff_fwd`` (triton_threshold_attention.py:489-519) w.r.t.
    q1, q2, k1, k2, v and lambda: branch 1 with dout, branch 2 with
    -clamp(lambda) * dout, dv summed, and d lambda = -sum(out2 * dout) where
    torch.clamp passes the gradient (0 <= lambda <= 1), else 0."""
    lam = float(lambda_param)
    lamc = min(max(lam, 0.0), 1.0)
    dout = np.asarray(dout, dtype=dtype)
    dq1, dk1, dv1 = rect_bwd(q1, k1, v, dout, beta, relu_power_, normalize, dtype)
    dq2, dk2, dv2 = rect_bwd(q2, k2, v, -dtype(lamc) * dout, beta, relu_power_, normalize, dtype)
    if 0.0 <= lam <= 1.0:
        o2 = rect_fwd(q2, k2, v, beta, relu_power_, normalize, dtype)
        dlam = -float(np.sum(o2 * dout))
    else:
        dlam = 0.0
    return dq1, dq2, dk1, dk2, dv1 + dv2, dlam


def rel_l2(a, b) -> float:
    """||a - b||_2 / ||b||_2 over all entries, in float64 (NaN entries of b, i.e.
    rows outside a sample, are skipped)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    m = ~np.isnan(b)
    num = np.linalg.norm((a - b)[m])
    den = np.linalg.norm(b[m])
    if den == 0.0:
        return float(num)
    return float(num / den)


def bf16_round(x) -> np.ndarray:
    """Round-to-nearest-even of float32 values to bfloat16, returned widened to
    float32 (the rounding torch applies in ``.to(torch.bfloat16)``)."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounding = ((u >> 16) & 1) + 0x7FFF
    u = ((u + rounding) >> 16) << 16
    out = (u & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(nan, np.float32(np.nan), out)


def bwd_flops(batch_heads: int, seq_len: int, head_dim: int, differential: bool) -> float:
    """Dense causal algorithmic FLOPs of the backward: per branch five GEMMs of
    2*S*S*D/2 per (batch, head) -- recomputed S, dP = dout V^T, dV = P^T dout,
    dQ = dA K, dK = dA^T Q -- twice for the differential form."""
    gemms = 10 if differential else 5
    return float(gemms) * float(batch_heads) * float(seq_len) ** 2 * float(head_dim)


def flops(batch_heads: int, seq_len: int, head_dim: int, differential: bool) -> float:
    """Dense causal algorithmic FLOPs: 2 (rect) or 3 (diff) GEMMs of
    2*S*S*D/2 per (batch, head)."""
    gemms = 3 if differential else 2
    return float(gemms) * float(batch_heads) * float(seq_len) ** 2 * float(head_dim)
