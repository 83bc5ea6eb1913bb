"""O(T)-state SPD delta rule in head-major layout -- drop-in for ``kata/spd/chunk_state_v2.py``.

Same public names and signatures as the reference module:
  flash_delta_state(q, k, v, beta, M, scale=None, C=64) -> o                          (:385-387)
  _StateDelta                                                                          (:354-382)
  spd_delta_state_v2(q, k, v, beta, M, scale=None, C=64, DVB=None, BI=None,
                     return_us=False) -> o or (o, U, S)                                 (:304-351)
  spd_delta_state_bwd(q, k, v, beta, do, U, S_final, M, scale=None, C=64, BI=None)
                     -> (dq, dk, dv, dbeta)                                             (:770-813)

q, k, v are head-major (B, H, T, D), beta (B, H, T); o, U are fp32 (B, H, T, DV) and S is the fp32
final state (B*H, E*E, DV), S = sum_t psi(k_t) U_t^T with psi(x)[a,b] = scale sum_g x_{g,a} x_{g,b}.
The function is the raw-numerator delta rule of ``flash_delta`` (normalize=False); it runs on the
same library entry points (``kata_delta_fwd`` / ``kata_delta_bwd``), whose U and state come from an
O(T) chunk scan over the feature state.  DVB and BI (Triton tiling knobs) are accepted and ignored.
"""

from __future__ import annotations

import torch

from .flash_delta import _bwd_call, _fwd_call

__all__ = ["flash_delta_state", "spd_delta_state_v2", "spd_delta_state_bwd"]


def _tm(x):
    return None if x is None else x.transpose(1, 2).contiguous()


def _hm(x):
    return x.transpose(1, 2).contiguous()


def spd_delta_state_v2(q, k, v, beta, M, scale=None, C=64, DVB=None, BI=None, return_us=False):
    B, H, T, D = q.shape
    DV = v.shape[-1]
    E = D // M
    S = torch.empty(B * H, E * E, DV, device=q.device, dtype=torch.float32) if return_us else None
    U, o, _ = _fwd_call(_tm(q), _tm(k), _tm(v), _tm(beta), M, scale, False, 0.0, phases=0, state=S)
    o = _hm(o)
    return (o, _hm(U), S) if return_us else o


def spd_delta_state_bwd(q, k, v, beta, do, U, S_final, M, scale=None, C=64, BI=None):
    """Gradients (fp32, head-major) of the raw numerator for upstream ``do``."""
    B, H, T, _ = q.shape
    z = torch.zeros(B, T, H, device=q.device, dtype=torch.float32)
    dq, dk, dv, db = _bwd_call(_tm(q), _tm(k), _tm(v), _tm(beta), _tm(U), _tm(do), M, scale, False, 0.0, z=z)
    return _hm(dq), _hm(dk), _hm(dv), db.transpose(1, 2).contiguous()


class _StateDelta(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, beta, M, scale, C):
        o, U, S = spd_delta_state_v2(q, k, v, beta, M, scale=scale, C=C, return_us=True)
        ctx.save_for_backward(q, k, v, beta, U, S)
        ctx.M, ctx.scale, ctx.C = M, scale, C
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, beta, U, S = ctx.saved_tensors
        dq, dk, dv, db = spd_delta_state_bwd(q, k, v, beta, do, U, S, ctx.M, scale=ctx.scale, C=ctx.C)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), db.to(beta.dtype), None, None, None


def flash_delta_state(q, k, v, beta, M, scale=None, C=64):
    """Trainable O(T)-state SPD delta (raw numerator, no normalisation), head-major."""
    return _StateDelta.apply(q, k, v, beta, M, scale, C)
