"""Recurrent (decode) form of causal KATA-SPD attention, concat score.

The reference has no decode path for the flash attention: its layer returns ``final_state=None``
from the flash branch (``kata/layer.py:293``, ``:374-376``, ``:532-537``), so generating a token
re-runs causal attention over the whole prefix.  Because the concat score is an inner product of
quadratic features, A[t,s] = psi(q_t) . psi(k_s) with psi(x)[g,a,b] = scale * x_{g,a} x_{g,b}
(F = M E^2 features per head), every prefix is summarised by the state

    [P | z] = sum_s psi(k_s) [v_s | 1]          (F x (Dv+1) per head, fp32)

and a token t after that prefix has

    o_t = (n_t + psi(q_t)^T P) / D_t',   D_t = d_t + psi(q_t)^T z,   x' = x if x > 0 else 1,

with n_t / d_t the causal numerator / denominator among the new tokens themselves.  This is the
combine step of the sequence-parallel path (``linatt_b200.sequence_parallel``) with the earlier
tokens in place of earlier ranks, so a step of one token or of a chunk costs O(F (Dv+1)) per head
and token instead of O(t).

Scope: concat score, H == HQ, no decay (as the sequence-parallel path).  Inference only (no
autograd).  The state's feature products are bf16 GEMMs with fp32 accumulation, so results match
``parallel_kata_attn`` over the whole sequence to bf16 accuracy.
"""

from __future__ import annotations

import torch

from . import parallel_kata_attn as pka
from .sequence_parallel import _features, _ldw, _scale, _v1, sp_forward_combine

__all__ = ["kata_attn_state", "kata_attn_step"]


def _check(q, k, v, num_groups):
    if q is not None and q.shape[:3] != k.shape[:3]:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} must share (B, T, H)")
    if k.shape[:3] != v.shape[:3]:
        raise ValueError(f"k {tuple(k.shape)} and v {tuple(v.shape)} must share (B, T, H)")
    if k.shape[-1] % num_groups:
        raise ValueError(f"head dim {k.shape[-1]} is not a multiple of num_groups={num_groups}")


@torch.no_grad()
def kata_attn_state(k, v, num_groups=4, scale=None):
    """State [P | z] = sum_s psi(k_s) [v_s | 1] of all tokens of k (B,T,H,D), v (B,T,H,Dv):
    an fp32 tensor (B*H, F, ldw), F = M (D/M)^2, columns [0,Dv) = P, column Dv = z, the rest 0."""
    _check(None, k, v, num_groups)
    scale = _scale(k.shape[-1], num_groups, scale)
    Rk = _features(k, num_groups, scale)
    return torch.bmm(Rk.transpose(1, 2), _v1(v, _ldw(v.shape[-1])), out_dtype=torch.float32)


@torch.no_grad()
def kata_attn_step(q, k, v, state=None, num_groups=4, scale=None, update_state=True):
    """Outputs for new tokens q, k (B,Tn,H,D), v (B,Tn,H,Dv) that follow the tokens summarised in
    ``state`` (None: no earlier tokens), and the state extended by them (``state`` itself when
    ``update_state`` is False).  o (B,Tn,H,Dv) in v's dtype equals the corresponding rows of
    ``parallel_kata_attn`` over the whole sequence."""
    _check(q, k, v, num_groups)
    scale = _scale(q.shape[-1], num_groups, scale)
    o_loc, den_loc = pka._fwd(q, k, v, num_groups, scale, "concat")
    o, _ = sp_forward_combine(q, o_loc, den_loc, state, num_groups, scale)
    if update_state:
        add = kata_attn_state(k, v, num_groups, scale)
        state = add if state is None else state + add
    return o, state
