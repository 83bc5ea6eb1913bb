"""Recurrent (decode) form of causal KATA-SPD attention, concat score.

The reference has no decode path for the flash attention: the quadratic-feature branch of its
layer (``kata/layer.py:421-492``) sets ``final_state = None``, so the layer cache stores no state
(``:532-537``) and generating a token re-runs causal attention over the whole prefix.  Because the concat score is an inner product of
quadratic features, A[t,s] = psi(q_t) . psi(k_s) with psi(x)[g,a,b] = scale * x_{g,a} x_{g,b}
(F = M E^2 features per head), every prefix is summarised by the state

    [P | z] = sum_s psi(k_s) [v_s | 1]          (F x (Dv+1) per head, fp32)

and a token t after that prefix has

    o_t = (n_t + psi(q_t)^T P) / D_t',   D_t = d_t + psi(q_t)^T z,   x' = x if x > 0 else 1,

with n_t / d_t the causal numerator / denominator among the new tokens themselves.  This is the
combine step of the sequence-parallel path (``linatt_b200.sequence_parallel``) with the earlier
tokens in place of earlier ranks, so a step of one token or of a chunk costs O(F (Dv+1)) per head
and token instead of O(t).  ``kata_attn_decode`` does the one-token generation step as a single
fused kernel (``kata_decode_step``): one pass over the fp32 state, updated in place.

Scope: concat score, H == HQ, no decay (as the sequence-parallel path).  Inference only (no
autograd).  The state's feature products are bf16 GEMMs with fp32 accumulation, so results match
``parallel_kata_attn`` over the whole sequence to bf16 accuracy.
"""

from __future__ import annotations

import torch

from . import _lib
from . import parallel_kata_attn as pka
from .sequence_parallel import _features, _ldw, _scale, _v1, sp_forward_combine

__all__ = ["kata_attn_state", "kata_attn_step", "kata_attn_decode"]

# Decode workspaces (per-head tickets + chunk partials), one per (device, stream).  A call leaves
# the tickets of its geometry zero, so a workspace is zeroed again only when the geometry changes
# (its ticket slots may then hold partials of the earlier geometry).
_work: dict[tuple[int, int], tuple[torch.Tensor, tuple]] = {}


def _workspace(dev, nbytes, geometry):
    key = (dev.index, _lib.stream_handle(dev))
    w, geo = _work.get(key, (None, None))
    if w is None or w.numel() < nbytes:
        w = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=dev)
    elif geo != geometry:
        w.zero_()
    _work[key] = (w, geometry)
    return w


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


@torch.no_grad()
def kata_attn_decode(q, k, v, state, num_groups=4, scale=None, return_den=False):
    """One generation step: q, k (B,H,D) or (B,1,H,D), v likewise with Dv, following the tokens
    summarised in ``state`` (B*H, F, ldw) fp32 -- as made by ``kata_attn_state`` -- which is
    updated IN PLACE to include this token.  Returns o in v's shape and dtype (and the
    denominator y (B,H) fp32 when ``return_den``): the token's row of ``parallel_kata_attn`` over
    the whole sequence.  One ``kata_decode_step`` kernel launch."""
    dev = _lib.require_cuda(q, k, v, state)
    shape = v.shape
    if q.dim() == 4:
        if q.shape[1] != 1 or k.shape[1] != 1 or v.shape[1] != 1:
            raise ValueError("kata_attn_decode takes one token; use kata_attn_step for chunks")
        q, k, v = q[:, 0], k[:, 0], v[:, 0]
    B, H, D = q.shape
    Dv = v.shape[-1]
    if k.shape != (B, H, D) or v.shape[:2] != (B, H):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if D % num_groups:
        raise ValueError(f"head dim {D} is not a multiple of num_groups={num_groups}")
    F = num_groups * (D // num_groups) ** 2
    if state.dtype != torch.float32 or state.dim() != 3 or state.shape[:2] != (B * H, F) or \
            state.shape[2] < Dv + 1 or not state.is_contiguous():
        raise ValueError(f"state must be contiguous fp32 (B*H, F, >=Dv+1) = ({B * H}, {F}, >={Dv + 1}), "
                         f"got {tuple(state.shape)} {state.dtype}")
    scale = _scale(D, num_groups, scale)
    dt = pka._common_dtype(q, k, v)
    qc, kc, vc = (x.to(dt).contiguous() for x in (q, k, v))
    lds = state.shape[2]
    L = _lib.lib()
    nbytes = L.kata_decode_workspace_bytes(B, H, D, Dv, num_groups, lds)
    if nbytes == 0:
        raise ValueError(f"unsupported decode geometry B={B} H={H} D={D} Dv={Dv} M={num_groups} lds={lds}")
    with torch.cuda.device(dev):
        work = _workspace(dev, nbytes, (B, H, D, Dv, num_groups, lds))
        o = torch.empty(B, H, Dv, device=dev, dtype=dt)
        den = torch.empty(B, H, device=dev, dtype=torch.float32) if return_den else None
        _lib.check(L.kata_decode_step(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), state.data_ptr(), o.data_ptr(),
                                      _lib.ptr(den), work.data_ptr(), _lib.DTYPE[dt], B, H, D, Dv, num_groups,
                                      lds, float(scale), _lib.stream_handle(dev)), "kata_decode_step")
    o = o.to(v.dtype).reshape(shape)
    return (o, den) if return_den else o
