"""PyTorch-fp32 restatement of the reference's CPU path -- TEST / BASELINE INFRASTRUCTURE ONLY.

Used by ``bench.py`` as the timed CPU baseline (``cpu_baseline.kind = "port"``) and as its
``--impl reference`` arm, and by tests as a second CPU witness.  It restates, operation for
operation, the reference's own PyTorch implementation of the hot path on CPU tensors:

  fwd -- ``_kata_decay_ref`` (kata/parallel_kata_attn.py:291-310): einsum of per-group dots,
         squared and summed, causal mask (decay factor exp(min(c_t-c_s,0)) when c is given),
         o = A v / (sum A + 1e-20)
  bwd -- ``parallel_kata_attn_bwd`` (kata/parallel_kata_attn.py:49-146): fp32 recompute of A,
         P = A / den, delta = <o, dO>, dV = P^T dO, dA = (dO V^T - delta)/den, da = 2 qk dA,
         dQ = scale da K, dK = scale da^T Q (MHA form)

The reference is not importable on the benchmark host, so this restatement is what runs there.
"""

from __future__ import annotations

import torch


def kata_fwd_ref(q, k, v, c, num_groups, scale):
    """o for (B,T,H,D) fp32 CPU tensors; c (B,T,H) or None (no decay)."""
    B, T, H, Kd = q.shape
    M = num_groups
    E = Kd // M
    qg = q.view(B, T, H, M, E)
    kg = k.view(B, T, H, M, E)
    qk = torch.einsum("bthme,bshme->bhtsm", qg, kg)
    A = ((scale * qk) ** 2).sum(-1)
    if c is not None:
        cH = c.transpose(1, 2)
        A = A * torch.exp(torch.clamp(cH[:, :, :, None] - cH[:, :, None, :], max=0.0))
    A = A * torch.tril(torch.ones(T, T, dtype=A.dtype))
    den = A.sum(-1)
    o = torch.einsum("bhts,bshd->bthd", A, v) / (den.transpose(1, 2)[..., None] + 1e-20)
    return o, den.transpose(1, 2).contiguous()


def kata_bwd_ref(q, k, v, o, den, do, num_groups, scale):
    """(dq, dk, dv) for the concat score, MHA (B,T,H,D) fp32 CPU tensors."""
    B, T, H, d_k = q.shape
    M = num_groups
    E = d_k // M
    Df = den.clamp_min(1e-12)
    qg = q.view(B, T, H, M, E)
    kg = k.view(B, T, H, M, E)
    qk = torch.einsum("bthme,bshme->bhtsm", qg, kg) * scale
    A = (qk * qk).sum(-1)
    causal = torch.tril(torch.ones(T, T, dtype=torch.bool))
    A = A * causal
    P = A / Df.permute(0, 2, 1).unsqueeze(-1)
    delta = (o * do).sum(-1).permute(0, 2, 1)
    do_p = do.permute(0, 2, 1, 3)
    dV = torch.einsum("bhts,bhtv->bhsv", P, do_p)
    dN_V = torch.einsum("bhtv,bhsv->bhts", do_p, v.permute(0, 2, 1, 3))
    dA = (dN_V - delta.unsqueeze(-1)) / Df.permute(0, 2, 1).unsqueeze(-1)
    dA = dA * causal
    da = 2.0 * qk * dA.unsqueeze(-1)
    dQ = scale * torch.einsum("bhtsm,bshme->bthme", da, kg)
    dK = scale * torch.einsum("bhtsm,bthme->bshme", da, qg)
    return dQ.reshape(B, T, H, d_k), dK.reshape(B, T, H, d_k), dV.permute(0, 2, 1, 3).contiguous()


def fwd_bwd_slice(q, k, v, do, num_groups, scale):
    """One full forward + backward of the reference CPU path (the unit the CPU baseline times)."""
    o, den = kata_fwd_ref(q, k, v, None, num_groups, scale)
    return kata_bwd_ref(q, k, v, o, den, do, num_groups, scale)
