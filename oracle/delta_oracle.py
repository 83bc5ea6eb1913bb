"""CPU oracle for the SPD delta rule ``flash_delta`` -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s CPU legs may import this module; the product path never does.

Restatement (float64 torch on CPU, one (batch, head) slice at a time) of
``kata/spd/flash_delta.py``:
  * kernel  kappa(x, y) = sum_{g,h} (scale * x_g . y_h)^2  (sum over all group pairs), with the
    reference's convention of applying s = sqrt(scale) to both operands (:193, :202): so
    (s x_g).(s y_h) = scale x_g.y_h; scale defaults to 1/E (E = D/M);
  * A_kk = kappa(k_t, k_s), A_qk = kappa(q_t, k_s)                       (:3-9)
  * U = (I + diag(beta) tril(A_kk, -1))^{-1} diag(beta) V                  (:1-9, K14 :27-183)
  * num = tril(A_qk) U (diagonal included)                                 (:975-985, K15)
  * normalize: den_t = sum_{s<=t} A_qk[t,s], o = num / (den + eps)         (:1049, :1062-1082)
  * the backward is the gradient of that function; the reference states its normalized backward
    is "consistent" (den propagates its gradient, :1111-1116), which autograd of this forward is.
The erase term E = tril(A_kk, -1) U (so that beta*(V - E) = U) is also returned, because the
backward uses it for d(beta).

Parity: ``tests/golden/make_golden_delta.py`` runs the reference's U solve (Triton K14, Triton CPU
interpreter) and pins this module at single-chunk size; the interpreter cannot run the
reference's bf16 tensor-core dots of the readout and backward, so this module is also checked
against fixtures that the reference's own Triton kernels produced on a B200
(``tests/golden/make_golden_delta_gpu.py``).
"""

from __future__ import annotations

import numpy as np
import torch


def _kappa(x, y, M, scale):
    """x (T,D), y (S,D) float64 -> (T,S) sum-score kernel."""
    T, D = x.shape
    E = D // M
    xg = x.reshape(T, M, E)
    yg = y.reshape(y.shape[0], M, E)
    ip = torch.einsum("tge,she->tsgh", xg, yg) * scale
    return (ip * ip).sum((-1, -2))


def _head(q, k, v, beta, M, scale, normalize, eps):
    T = q.shape[0]
    Akk = _kappa(k, k, M, scale)
    Aqk = _kappa(q, k, M, scale)
    L = torch.tril(Akk, -1)
    I = torch.eye(T, dtype=q.dtype)
    U = torch.linalg.solve_triangular(I + beta[:, None] * L, beta[:, None] * v, upper=False, unitriangular=True)
    P = torch.tril(Aqk)
    num = P @ U
    Em = L @ U
    den = P.sum(1)
    o = num / (den[:, None] + eps) if normalize else num
    return o, U, Em, den


def flash_delta(q, k, v, beta, M, scale=None, normalize=False, eps=1e-5, grad_out=None):
    """Time-major (B,T,H,D) inputs (any float arrays).  Returns a dict with o, U, E, den (float64
    numpy) and, when ``grad_out`` (B,T,H,Dv) is given, dq, dk, dv, dbeta."""
    q, k, v, beta = (torch.as_tensor(np.asarray(x), dtype=torch.float64) for x in (q, k, v, beta))
    B, T, H, D = q.shape
    if scale is None:
        scale = 1.0 / (D // M)
    want_grad = grad_out is not None
    if want_grad:
        go = torch.as_tensor(np.asarray(grad_out), dtype=torch.float64)
        q, k, v, beta = (x.clone().requires_grad_(True) for x in (q, k, v, beta))
    outs = {n: [] for n in ("o", "U", "E", "den")}
    total = 0.0
    for b in range(B):
        for h in range(H):
            o, U, Em, den = _head(q[b, :, h], k[b, :, h], v[b, :, h], beta[b, :, h], M, scale, normalize, eps)
            for n, x in zip(("o", "U", "E", "den"), (o, U, Em, den)):
                outs[n].append(x)
            if want_grad:
                total = total + (o * go[b, :, h]).sum()
    res = {}
    for n in ("o", "U", "E"):
        res[n] = torch.stack(outs[n]).reshape(B, H, T, -1).permute(0, 2, 1, 3).detach().numpy()
    res["den"] = torch.stack(outs["den"]).reshape(B, H, T).permute(0, 2, 1).detach().numpy()
    if want_grad:
        total.backward()
        res.update(dq=q.grad.numpy(), dk=k.grad.numpy(), dv=v.grad.numpy(), dbeta=beta.grad.numpy())
    return res


def state_lin(q, k, v, M, scale=None, grad_out=None):
    """Linear SPD numerator o = tril(kappa(q, k)) v and its gradients (float64), head-major
    (B, H, T, D) inputs, restating kata/spd/chunk_state_lin.py:1-12 (the chunked-state kernel
    computes exactly this raw numerator) and its backward (:437-504).  Returns a dict o [, dq, dk, dv]."""
    q, k, v = (torch.as_tensor(np.asarray(x), dtype=torch.float64) for x in (q, k, v))
    B, H, T, D = q.shape
    scale = 1.0 / (D // M) if scale is None else float(scale)
    want = grad_out is not None
    q, k, v = (x.clone().requires_grad_(want) for x in (q, k, v))
    o = torch.zeros(B, H, T, v.shape[-1], dtype=torch.float64)
    outs = []
    for b in range(B):
        for h in range(H):
            outs.append(torch.tril(_kappa(q[b, h], k[b, h], M, scale)) @ v[b, h])
    o = torch.stack(outs).reshape(B, H, T, -1)
    res = {"o": o.detach().numpy()}
    if want:
        o.backward(torch.as_tensor(np.asarray(grad_out), dtype=torch.float64))
        res.update(dq=q.grad.numpy(), dk=k.grad.numpy(), dv=v.grad.numpy())
    return res


def chunk_scan(q, k, v, M, scale=None, eps=1e-6):
    """Normalised sum-score forward of kata/spd/chunk_scan.py:295-406 (sum mode), head-major:
    den = max(sum_{s<=t} kappa, eps), o = tril(kappa) v / den (its output kernel, :166-177)."""
    q, k, v = (torch.as_tensor(np.asarray(x), dtype=torch.float64) for x in (q, k, v))
    B, H, T, D = q.shape
    scale = 1.0 / (D // M) if scale is None else float(scale)
    o = torch.zeros(B, H, T, v.shape[-1], dtype=torch.float64)
    den = torch.zeros(B, H, T, dtype=torch.float64)
    for b in range(B):
        for h in range(H):
            P = torch.tril(_kappa(q[b, h], k[b, h], M, scale))
            d = P.sum(1).clamp_min(eps)
            o[b, h] = (P @ v[b, h]) / d[:, None]
            den[b, h] = d
    return {"o": o.numpy(), "den": den.numpy()}
