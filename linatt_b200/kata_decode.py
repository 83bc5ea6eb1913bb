"""Recurrent (decode) form of causal KATA-SPD attention: concat and sum scores, decay, GQA.

The reference has no decode path for the flash attention: the quadratic-feature branch of its
layer (``kata/layer.py:421-492``) sets ``final_state = None``, so the layer cache stores no state
(``:532-537``) and generating a token re-runs causal attention over the whole prefix.  Both scores
are inner products of quadratic features, A[t,s] = psi(q_t) . psi(k_s) (E = D/M):

    concat  psi(x)[g,a,b] = scale * x_{g,a} x_{g,b}          F = M E^2
    sum     psi(x)[a,b]   = scale * sum_g x_{g,a} x_{g,b}    F = E^2

so a prefix is summarised by the state

    [P | z] = sum_s w_s psi(k_s) [v_s | 1]          (F x ldw per head, fp32)

(w_s = 1; with decay w_s = exp(c_t - c_s) for the current token t), and a token t after that
prefix has

    o_t = (n_t + psi(q_t)^T P) / D_t',   D_t = d_t + psi(q_t)^T z,   x' = x if x > 0 else 1,

with n_t / d_t the causal numerator / denominator among the new tokens themselves.  Without decay
the state is per key/value head and shared by its query heads (GQA); with decay it is per query
head.  ``kata_attn_decode`` does the one-token generation step as one fused kernel
(``kata_decode_step``): one pass over the fp32 state, updated in place.  ``kata_attn_step`` takes a
chunk of new tokens: the flash forward over the chunk, combined with psi(q)^T S.

Decay takes the per-token log-decay g_t = c_t - c_{t-1} (the layer's -exp(A_log) softplus(dt),
``kata/layer.py:440-447``); the recurrence S_t = exp(g_t) S_{t-1} + psi(k_t)[v_t|1] equals the
reference's factor exp(min(c_t - c_s, 0)) whenever c is non-increasing (g <= 0), as the layer's c is.
Inference only (no autograd).
"""

from __future__ import annotations

import torch

from . import _lib
from . import parallel_kata_attn as pka
from .sequence_parallel import _features, _ldw, _scale, _v1

__all__ = ["kata_attn_state", "kata_attn_step", "kata_attn_decode", "state_features"]

# Decode workspaces (per-state tickets + chunk partials), one per (device, stream).  A call leaves
# the tickets of its geometry zero, so a workspace is zeroed again only when the geometry changes
# (its ticket slots may then hold partials of the earlier geometry).
_workspaces: dict[tuple[int, int], tuple[torch.Tensor, tuple]] = {}


def _workspace(dev, nbytes, geometry):
    key = (dev.index, _lib.stream_handle(dev))
    w, geo = _workspaces.get(key, (None, None))
    if w is None or w.numel() < nbytes:
        w = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=dev)
    elif geo != geometry:
        w.zero_()
    _workspaces[key] = (w, geometry)
    return w


def _check_score(score, c):
    if score not in ("concat", "sum"):
        raise ValueError(f"score must be 'concat' or 'sum', got {score!r}")
    if c is not None and score != "concat":
        raise ValueError("decay pairs with the concat score only (as in the reference)")


def state_features(x, num_groups, scale, score="concat"):
    """psi(x) of x (B,T,H,D): (B*H, T, F) bf16 (head-major), by the feature kernels
    (``kata_sp_features`` / ``kata_sum_features``) when E = D/M is a multiple of 8."""
    if score == "concat":
        return _features(x, num_groups, scale)
    B, T, H, D = x.shape
    E = D // num_groups
    if E % 8 == 0:
        dev = _lib.require_cuda(x)
        xc = x.contiguous()
        R = torch.empty(B * H, T, E * E, device=dev, dtype=torch.bfloat16)
        _lib.check(_lib.lib().kata_sum_features(xc.data_ptr(), R.data_ptr(), _lib.DTYPE[xc.dtype], B, T, H, D,
                                                num_groups, float(scale), _lib.stream_handle(dev)),
                   "kata_sum_features")
        return R
    xg = x.float().view(B, T, H, num_groups, E)
    R = torch.einsum("bthga,bthgc->bhtac", xg, xg).mul_(scale)
    return R.reshape(B * H, T, E * E).to(torch.bfloat16)


@torch.no_grad()
def kata_attn_state(k, v, num_groups=4, scale=None, score="concat", c=None, HQ=None):
    """State of all tokens of k (B,T,H,D), v (B,T,H,Dv): fp32 (B*HS, F, ldw), columns [0,Dv) = P,
    column Dv = z, the rest 0.  Without decay HS = H.  With decay, c (B,T,HQ) is the cumulative
    log-decay, the rows are weighted by exp(c_last - c_s) and HS = HQ (the state is per query head)."""
    _check_score(score, c)
    B, T, H, D = k.shape
    if k.shape[:3] != v.shape[:3]:
        raise ValueError(f"k {tuple(k.shape)} and v {tuple(v.shape)} must share (B, T, H)")
    if D % num_groups:
        raise ValueError(f"head dim {D} is not a multiple of num_groups={num_groups}")
    scale = _scale(D, num_groups, scale)
    V1 = _v1(v, _ldw(v.shape[-1]))
    G = 1
    if c is not None:
        HQ = c.shape[2] if HQ is None else HQ
        if c.shape != (B, T, HQ) or HQ % H:
            raise ValueError(f"c must be (B, T, HQ) with HQ a multiple of H={H}, got {tuple(c.shape)}")
        G = HQ // H
        w = torch.exp(c[:, -1:, :].float() - c.float())  # (B, T, HQ)
        w = w.permute(0, 2, 1).reshape(B, H, G, T, 1)
        V1 = (V1.view(B, H, 1, T, -1).float() * w).to(torch.bfloat16).reshape(B * HQ, T, -1)
    E = D // num_groups
    ldw = V1.shape[-1]
    tc = (k.dtype in (torch.bfloat16, torch.float16) and E in (16, 32) and ldw <= 144
          and (num_groups <= 4 if score == "sum" else D in (64, 128)))
    if tc:  # psi(K)^T V1 on the tensor cores, psi formed in shared memory (kata_sp_state)
        F = E * E if score == "sum" else num_groups * E * E
        kc = k.contiguous()
        S = torch.empty(B * H * G, F, ldw, device=k.device, dtype=torch.float32)
        _lib.check(_lib.lib().kata_sp_state(kc.data_ptr(), V1.data_ptr(), S.data_ptr(), _lib.DTYPE[k.dtype], B, T, H,
                                            G, D, num_groups, _lib.SCORE[score], ldw, float(scale), 0, ldw,
                                            _lib.status_word(k.device).data_ptr(), _lib.stream_handle(k.device)),
                   "kata_sp_state")
        return S
    Rk = state_features(k, num_groups, scale, score)
    if G > 1:
        Rk = Rk.view(B, H, 1, T, -1).expand(B, H, G, T, Rk.shape[-1]).reshape(B * H * G, T, -1)
    return torch.bmm(Rk.transpose(1, 2), V1, out_dtype=torch.float32)


def _combine(q, o_loc, den_loc, XY):
    """o = (o_loc den_loc' + X) / D', D = den_loc + y (per query head; XY (B*HQ, T, ldw))."""
    B, T, HQ, Dv = o_loc.shape
    o = torch.empty_like(o_loc)
    D = torch.empty_like(den_loc)
    _lib.check(_lib.lib().kata_sp_combine(o_loc.data_ptr(), den_loc.data_ptr(), XY.data_ptr(), o.data_ptr(),
                                          D.data_ptr(), _lib.DTYPE[o_loc.dtype], B, T, HQ, Dv, XY.shape[-1],
                                          _lib.stream_handle(q.device)), "kata_sp_combine")
    return o, D


@torch.no_grad()
def kata_attn_step(q, k, v, state=None, num_groups=4, scale=None, score="concat", g=None, update_state=True):
    """Outputs for new tokens q (B,Tn,HQ,D), k (B,Tn,H,D), v (B,Tn,H,Dv) that follow the tokens
    summarised in ``state`` (None: no earlier tokens), and the state extended by them (``state``
    itself when ``update_state`` is False).  ``g`` (B,Tn,HQ): per-token log-decays (decay form).
    o (B,Tn,HQ,Dv) in v's dtype equals the corresponding rows of the full causal attention."""
    _check_score(score, g)
    B, Tn, HQ, D = q.shape
    H = k.shape[2]
    if k.shape[:2] != (B, Tn) or v.shape[:3] != k.shape[:3] or HQ % H:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    scale = _scale(D, num_groups, scale)
    c = None if g is None else torch.cumsum(g.float(), dim=1)  # chunk-local cumulative log-decay
    o_loc, den_loc = pka._fwd(q, k, v, num_groups, scale, score, c)
    o = o_loc
    if state is not None:
        Rq = state_features(q, num_groups, scale, score)  # (B*HQ, Tn, F)
        if c is None:  # the G query heads of a key/value head share its state
            XY = torch.bmm(Rq.view(B * H, (HQ // H) * Tn, -1), state.to(torch.bfloat16), out_dtype=torch.float32)
            XY = XY.view(B * HQ, Tn, -1)
        else:
            XY = torch.bmm(Rq, state.to(torch.bfloat16), out_dtype=torch.float32)
            XY *= torch.exp(c).permute(0, 2, 1).reshape(B * HQ, Tn, 1)
        o, _ = _combine(q, o_loc, den_loc, XY)
    if update_state:
        add = kata_attn_state(k, v, num_groups, scale, score, c, HQ)
        if state is None:
            state = add
        elif c is None:
            state = state + add
        else:
            state = state * torch.exp(c[:, -1, :]).reshape(B * HQ, 1, 1) + add
    return o, state


@torch.no_grad()
def kata_attn_decode(q, k, v, state, num_groups=4, scale=None, score="concat", g=None, return_den=False):
    """One generation step: q (B,HQ,D) or (B,1,HQ,D), k (B,H,D) / v (B,H,Dv) (or with the token
    axis), following the tokens summarised in ``state`` -- as made by ``kata_attn_state`` -- which
    is updated IN PLACE to include this token.  ``g`` (B,HQ): the token's log-decay (decay form;
    the state is then per query head).  Returns o in q's token layout with Dv and v's dtype (and
    the denominator (B,HQ) fp32 when ``return_den``): the token's row of the full causal attention.
    One ``kata_decode_step`` kernel launch."""
    _check_score(score, g)
    dev = _lib.require_cuda(q, k, v, state, g)
    tok = q.dim() == 4
    if tok:
        if q.shape[1] != 1 or k.shape[1] != 1 or v.shape[1] != 1:
            raise ValueError("kata_attn_decode takes one token; use kata_attn_step for chunks")
        q, k, v = q[:, 0], k[:, 0], v[:, 0]
        if g is not None and g.dim() == 3:
            g = g[:, 0]
    B, HQ, D = q.shape
    H, Dv = k.shape[1], v.shape[-1]
    if k.shape != (B, H, D) or v.shape[:2] != (B, H) or HQ % H:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if D % num_groups:
        raise ValueError(f"head dim {D} is not a multiple of num_groups={num_groups}")
    E = D // num_groups
    F = E * E if score == "sum" else num_groups * E * E
    HS = HQ if g is not None else H
    if state.dtype != torch.float32 or state.dim() != 3 or state.shape[:2] != (B * HS, F) or \
            state.shape[2] < Dv + 1 or not state.is_contiguous():
        raise ValueError(f"state must be contiguous fp32 (B*HS, F, >=Dv+1) = ({B * HS}, {F}, >={Dv + 1}), "
                         f"got {tuple(state.shape)} {state.dtype}")
    if g is not None and g.shape != (B, HQ):
        raise ValueError(f"g must be (B, HQ) = ({B}, {HQ}), got {tuple(g.shape)}")
    scale = _scale(D, num_groups, scale)
    dt = pka._common_dtype(q, k, v)
    qc, kc, vc = (x.to(dt).contiguous() for x in (q, k, v))
    gc = None if g is None else g.float().contiguous()
    lds = state.shape[2]
    with torch.cuda.device(dev):
        o = torch.empty(B, HQ, Dv, device=dev, dtype=dt)
        den = torch.empty(B, HQ, device=dev, dtype=torch.float32) if return_den else None
        a = _lib.DecodeArgs(q=qc.data_ptr(), k=kc.data_ptr(), v=vc.data_ptr(), g=_lib.ptr(gc),
                            state=state.data_ptr(), o=o.data_ptr(), den=_lib.ptr(den), work=None,
                            dtype=_lib.DTYPE[dt], B=B, HQ=HQ, H=H, D=D, Dv=Dv, M=num_groups, lds=lds,
                            score=_lib.SCORE[score], scale=float(scale))
        L = _lib.lib()
        nbytes = L.kata_decode_workspace_bytes(a)
        if nbytes == 0:
            raise ValueError(f"unsupported decode geometry B={B} HQ={HQ} H={H} D={D} Dv={Dv} M={num_groups} "
                             f"lds={lds} score={score}")
        a.work = _workspace(dev, nbytes, (B, HQ, H, D, Dv, num_groups, lds, score, g is None)).data_ptr()
        _lib.check(L.kata_decode_step(a, _lib.stream_handle(dev)), "kata_decode_step")
    o = o.to(v.dtype)
    if tok:
        o = o.unsqueeze(1)
    return (o, den) if return_den else o
