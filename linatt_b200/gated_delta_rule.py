"""Gated delta rule (GDN) -- drop-in for ``fla.ops.gated_delta_rule`` as the reference uses it.

The reference's gated_deltanet models call fla's ``chunk_gated_delta_rule``
(``fla/ops/gated_delta_rule/chunk.py:365-526``; fla is third-party, pinned 0.5.0 by
``scripts/setup.sh:27``) through ``fla/layers/gated_deltanet.py:266-278``.  This module provides
the same entry point, argument for argument:

  chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None,
                         output_final_state=False, use_qk_l2norm_in_kernel=False,
                         cu_seqlens=None, cu_seqlens_cpu=None, cp_context=None,
                         transpose_state_layout=False, **kwargs) -> (o, final_state)

with ``kwargs`` use_gate_in_kernel / A_log / dt_bias (g <- -exp(A_log) softplus(g + dt_bias)),
plus ``ChunkGatedDeltaRuleFunction`` and the alias ``chunk_gdn``.  All recurrence arithmetic runs
in ``libkata_b200.so`` (``kata_gdn_fwd`` / ``kata_gdn_bwd``).  The q/k l2norm and the in-kernel
gate are applied as differentiable torch prologues before the library call.  Context parallelism
(``cp_context``) is fla's own multi-GPU scheme and is not provided.  The kernels work on 64-wide
heads; narrower q/k/v heads are zero-padded to 64 (exact); value heads wider than 64 run as
independent 64-column slices of the state (exact, see ``_value_slices``); key heads wider than 64
are not supported.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib

__all__ = ["chunk_gated_delta_rule", "chunk_gdn", "ChunkGatedDeltaRuleFunction", "fused_recurrent_gated_delta_rule",
           "fused_recurrent_gdn"]

CHUNK = 64

# Kernel family of every call ("auto" | "tc" | "simt"): auto runs the tcgen05 kernels for bf16 / fp16
# inputs and the fp32-exact CUDA-core kernels for fp32 inputs.  Tests switch it to run one family.
ALGO = "auto"


def _dtype(*ts):
    dt = ts[0].dtype
    for t in ts[1:]:
        dt = torch.promote_types(dt, t.dtype)
    if dt not in _lib.DTYPE:
        raise TypeError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16")
    return dt


def _chunk_tables(cu_seqlens, cu_seqlens_cpu, B, T, dev):
    """(N, num_chunks, cu int32 device or None, chunk offsets int32 device or None)."""
    if cu_seqlens is None:
        return B, B * ((T + CHUNK - 1) // CHUNK), None, None
    cs = (cu_seqlens_cpu if cu_seqlens_cpu is not None else cu_seqlens.cpu()).to(torch.int64)
    lens = cs[1:] - cs[:-1]
    co = torch.zeros(len(lens) + 1, dtype=torch.int64)
    co[1:] = torch.cumsum((lens + CHUNK - 1) // CHUNK, 0)
    return (len(lens), int(co[-1]), cu_seqlens.to(device=dev, dtype=torch.int32).contiguous(),
            co.to(device=dev, dtype=torch.int32))


KDIM = 64  # key / value width of the kernels; narrower heads are zero-padded (exact)


def _pad_last(x, n):
    return x if x is None or x.shape[-1] == n else F.pad(x, (0, n - x.shape[-1]))


def _pad_state(h):
    if h is None or (h.shape[-2] == KDIM and h.shape[-1] == KDIM):
        return h
    return F.pad(h, (0, KDIM - h.shape[-1], 0, KDIM - h.shape[-2])).contiguous()


def _check_width(K, V):
    if K > KDIM or V > KDIM:
        raise NotImplementedError(f"linatt_b200 gated delta rule covers head widths up to {KDIM} (got K={K}, V={V})")


def _value_slices(V):
    """Value-column ranges of at most KDIM.  Every value column of the state S (K x V) follows its
    own recurrence S[:, j] <- e^g (I - beta k k^T) S[:, j] + beta v_j k, and o[j] = S[:, j] . q, so a
    head wider than the kernels runs as independent slices of the value dimension whose q, k, g and
    beta gradients add up (fla's chunk_gated_delta_rule, chunk.py:365, accepts any V)."""
    return [(s0, min(s0 + KDIM, V)) for s0 in range(0, V, KDIM)]


def _fwd_sliced(q, k, v, g, beta, scale, h0, want_final, tables):
    """_fwd over value slices of at most KDIM columns: (o, A, final state, [forward workspace per slice])."""
    if v.shape[-1] <= KDIM:
        o, A, ht, ws = _fwd(q, k, v, g, beta, scale, h0, want_final, tables)
        return o, A, ht, [ws]
    os_, hts, wss, A = [], [], [], None
    for s0, s1 in _value_slices(v.shape[-1]):
        h0s = None if h0 is None else h0[..., s0:s1].contiguous()
        o, A, ht, ws = _fwd(q, k, v[..., s0:s1].contiguous(), g, beta, scale, h0s, want_final, tables)
        os_.append(o)
        hts.append(ht)
        wss.append(ws)
    ht = torch.cat(hts, -1) if want_final else None
    return torch.cat(os_, -1), A, ht, wss


def _bwd_sliced(q, k, v, g, beta, A, scale, h0, do, dht, tables, fwd_ws, grad16=False):
    """_bwd over the value slices of _fwd_sliced (fwd_ws: one workspace per slice)."""
    if v.shape[-1] <= KDIM:
        return _bwd(q, k, v, g, beta, A, scale, h0, do, dht, tables, fwd_ws=fwd_ws[0], grad16=grad16)
    acc, dvs, dh0s = None, [], []
    for (s0, s1), ws in zip(_value_slices(v.shape[-1]), fwd_ws):
        h0s = None if h0 is None else h0[..., s0:s1].contiguous()
        dhts = None if dht is None else dht[..., s0:s1].contiguous()
        dq, dk, dv, dg, db, dh0 = _bwd(q, k, v[..., s0:s1].contiguous(), g, beta, A, scale, h0s,
                                       do[..., s0:s1].contiguous(), dhts, tables, fwd_ws=ws)
        part = [x.float() for x in (dq, dk, dg, db)]
        acc = part if acc is None else [a + b for a, b in zip(acc, part)]
        dvs.append(dv)
        dh0s.append(dh0)
    dq, dk, dg, db = acc
    return dq, dk, torch.cat(dvs, -1), dg, db, (None if h0 is None else torch.cat(dh0s, -1))


def _fwd(q, k, v, g, beta, scale, h0, want_final, tables):
    dev = _lib.require_cuda(q, k, v, g, beta, h0)
    K0, V0 = q.shape[-1], v.shape[-1]
    _check_width(K0, V0)  # V0 <= KDIM here: wider value heads arrive as slices (_fwd_sliced)
    q, k, v = (_pad_last(x, KDIM).contiguous() for x in (q, k, v))
    h0 = _pad_state(h0)
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    N, NC, cu, co = tables
    dt = _dtype(q, k, v)
    o = torch.empty(B, T, HV, V, device=dev, dtype=dt)
    A = torch.empty(B, T, HV, CHUNK, device=dev, dtype=torch.float32)
    ht = torch.empty(N, HV, K, V, device=dev, dtype=torch.float32) if want_final else None
    a = _lib.GdnFwdArgs(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), g=g.data_ptr(), beta=beta.data_ptr(), h0=_lib.ptr(h0),
        o=o.data_ptr(), ht=_lib.ptr(ht), A=A.data_ptr(), cu_seqlens=_lib.ptr(cu), chunk_offsets=_lib.ptr(co),
        workspace=None, workspace_bytes=0, dtype=_lib.DTYPE[dt], B=B, T=T, H=H, HV=HV, K=K, V=V, N=N,
        num_chunks=NC, scale=float(scale), algo=_lib.ALGO[ALGO])
    L = _lib.lib()
    ws = torch.empty(int(L.kata_gdn_fwd_workspace_bytes(a)), device=dev, dtype=torch.uint8)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(dev):
        _lib.check(L.kata_gdn_fwd(a, _lib.stream_handle(dev)), "kata_gdn_fwd")
    if V0 != V:
        o = o[..., :V0]
    if ht is not None and (K0 != K or V0 != V):
        ht = ht[..., :K0, :V0].contiguous()
    return o, A, ht, ws


def _bwd(q, k, v, g, beta, A, scale, h0, do, dht, tables, fwd_ws=None, grad16=False):
    dev = _lib.require_cuda(q, k, v, g, beta, A, h0, do, dht)
    K0, V0 = q.shape[-1], v.shape[-1]
    dt = _dtype(q, k, v)
    q, k, v = (_pad_last(x, KDIM).contiguous() for x in (q, k, v))
    h0 = _pad_state(h0)
    do = _pad_last(do.to(dt), KDIM).contiguous()
    dht = _pad_state(None if dht is None else dht.float())
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    N, NC, cu, co = tables
    f32 = dict(device=dev, dtype=torch.float32)
    # 16-bit gradients straight from the tensor-core kernels (no fp32 round trip) when they run and no
    # value-head group accumulates into a shared q/k head
    grad16 = grad16 and dt != torch.float32 and ALGO != "simt" and HV == H
    gq = dict(device=dev, dtype=dt if grad16 else torch.float32)
    dq = torch.empty(B, T, H, K, **gq)
    dk = torch.empty(B, T, H, K, **gq)
    dv = torch.empty(B, T, HV, V, **gq)
    dg = torch.empty(B, T, HV, **f32)
    db = torch.empty(B, T, HV, **f32)
    dh0 = torch.empty(N, HV, K, V, **f32) if h0 is not None else None
    dht = None if dht is None else dht.float().contiguous()
    a = _lib.GdnBwdArgs(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), g=g.data_ptr(), beta=beta.data_ptr(), h0=_lib.ptr(h0),
        A=A.data_ptr(), dout=do.data_ptr(), dht=_lib.ptr(dht), dq=dq.data_ptr(), dk=dk.data_ptr(),
        dv=dv.data_ptr(), dg=dg.data_ptr(), dbeta=db.data_ptr(), dh0=_lib.ptr(dh0), cu_seqlens=_lib.ptr(cu),
        chunk_offsets=_lib.ptr(co), workspace=None, workspace_bytes=0, fwd_workspace=_lib.ptr(fwd_ws),
        dtype=_lib.DTYPE[dt], B=B, T=T, H=H, HV=HV, K=K, V=V, N=N, num_chunks=NC, scale=float(scale),
        algo=_lib.ALGO[ALGO], grad_dtype=_lib.DTYPE[dt] if grad16 else 0)
    L = _lib.lib()
    ws = torch.empty(int(L.kata_gdn_bwd_workspace_bytes(a)), device=dev, dtype=torch.uint8)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(dev):
        _lib.check(L.kata_gdn_bwd(a, _lib.stream_handle(dev)), "kata_gdn_bwd")
    if K0 != K or V0 != V:
        dq, dk, dv = dq[..., :K0], dk[..., :K0], dv[..., :V0]
        dh0 = None if dh0 is None else dh0[..., :K0, :V0]
    return dq, dk, dv, dg, db, dh0


class ChunkGatedDeltaRuleFunction(torch.autograd.Function):
    """Same argument list as fla's ChunkGatedDeltaRuleFunction (chunk.py:238-362); the l2norm and
    gate options arrive already applied by ``chunk_gated_delta_rule``."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens=None,
                cu_seqlens_cpu=None, use_qk_l2norm_in_kernel=False, cp_context=None, transpose_state_layout=False,
                use_gate_in_kernel=False, A_log=None, dt_bias=None):
        if cp_context is not None:
            raise NotImplementedError("cp_context (fla context parallelism) is not provided by linatt_b200")
        B, T = q.shape[:2]
        dt = _dtype(q, k, v)
        qc, kc, vc = (x.to(dt).contiguous() for x in (q, k, v))
        gc, bc = g.float().contiguous(), beta.float().contiguous()
        h0 = None
        if initial_state is not None:
            h0 = initial_state.float()
            h0 = (h0.transpose(-1, -2) if transpose_state_layout else h0).contiguous()
        tables = _chunk_tables(cu_seqlens, cu_seqlens_cpu, B, T, q.device)
        if q.shape[-1] > KDIM:
            _check_width(q.shape[-1], v.shape[-1])
        o, A, ht, ws = _fwd_sliced(qc, kc, vc, gc, bc, scale, h0, output_final_state, tables)
        if ht is not None and transpose_state_layout:
            ht = ht.transpose(-1, -2).contiguous()
        # Besides fla's saved set (q, k, v, g, beta, A, initial state) the forward's workspace (chunk
        # states, u, W, U0, gamma) is kept, so the backward does not recompute the forward scan.
        ctx.save_for_backward(qc, kc, vc, gc, bc, A, h0, *ws)
        ctx.tables = tables
        ctx.scale = scale
        ctx.transpose_state_layout = transpose_state_layout
        ctx.dtypes = (q.dtype, k.dtype, v.dtype, g.dtype, beta.dtype,
                      None if initial_state is None else initial_state.dtype)
        return o.to(q.dtype), ht

    @staticmethod
    def backward(ctx, do, dht):
        qc, kc, vc, gc, bc, A, h0, *ws = ctx.saved_tensors
        if dht is not None and ctx.transpose_state_layout:
            dht = dht.transpose(-1, -2)
        tq, tk, tv, tg, tb, th = ctx.dtypes
        same = tq == tk == tv == qc.dtype
        dq, dk, dv, dg, db, dh0 = _bwd_sliced(qc, kc, vc, gc, bc, A, ctx.scale, h0, do, dht, ctx.tables, ws,
                                              grad16=same)
        if dh0 is not None:
            dh0 = (dh0.transpose(-1, -2) if ctx.transpose_state_layout else dh0).to(th)
        return (dq.to(tq), dk.to(tk), dv.to(tv), dg.to(tg), db.to(tb), None, dh0, None, None, None, None, None,
                None, None, None, None)


def _l2norm(x):
    # fla/modules/l2norm.py:42,140: y = x / sqrt(sum(x^2) + 1e-6), computed in fp32, returned in x.dtype
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) + 1e-6)).to(x.dtype)


def chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None, output_final_state=False,
                           use_qk_l2norm_in_kernel=False, cu_seqlens=None, cu_seqlens_cpu=None, cp_context=None,
                           transpose_state_layout=False, **kwargs):
    """Returns (o (B,T,HV,V) in q's dtype, final_state (N,HV,K,V) fp32 or None)."""
    if q.shape[2] != k.shape[2]:
        raise ValueError(f"q and k must have the same number of heads, got {q.shape[2]} and {k.shape[2]}")
    H, HV = q.shape[2], v.shape[2]
    if HV % H != 0:
        raise ValueError(f"num_v_heads (HV={HV}) must be divisible by num_heads (H={H})")
    if "head_first" in kwargs:
        raise DeprecationWarning("head_first has been removed. Inputs must be in `[B, T, H, ...]` format.")
    if cp_context is not None:
        raise NotImplementedError("cp_context (fla context parallelism) is not provided by linatt_b200")
    if cu_seqlens is not None:
        if q.shape[0] != 1:
            raise ValueError(f"The batch size is expected to be 1 rather than {q.shape[0]} when using `cu_seqlens`.")
        if initial_state is not None and initial_state.shape[0] != len(cu_seqlens) - 1:
            raise ValueError(f"The number of initial states is expected to be equal to the number of input "
                             f"sequences, i.e., {len(cu_seqlens) - 1} rather than {initial_state.shape[0]}.")
    if kwargs.get("use_gate_in_kernel", False):
        A_log, dt_bias = kwargs.get("A_log"), kwargs.get("dt_bias")
        assert A_log is not None, "A_log must be provided when use_gate_in_kernel=True."
        x = g.float() + (dt_bias.float() if dt_bias is not None else 0.0)
        g = -A_log.float().exp() * F.softplus(x)
    if use_qk_l2norm_in_kernel:
        q, k = _l2norm(q), _l2norm(k)
    if scale is None:
        scale = k.shape[-1] ** -0.5
    return ChunkGatedDeltaRuleFunction.apply(q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens,
                                             cu_seqlens_cpu, False, None, transpose_state_layout, False, None, None)


chunk_gdn = chunk_gated_delta_rule


def fused_recurrent_gated_delta_rule(q, k, v, g=None, gk=None, gv=None, beta=None, scale=None, initial_state=None,
                                     output_final_state=False, use_qk_l2norm_in_kernel=False,
                                     use_gate_in_kernel=False, A_log=None, dt_bias=None, cu_seqlens=None,
                                     transpose_state_layout=False):
    """fla's token-recurrent entry point (``fla/ops/gated_delta_rule/fused_recurrent.py``), used by
    ``GatedDeltaNet`` in its ``fused_recurrent`` mode.  The recurrence is the same, so it runs on
    the chunked kernels; the per-key / per-value gates ``gk`` / ``gv`` are not provided."""
    if gk is not None or gv is not None:
        raise NotImplementedError("linatt_b200: per-key / per-value gates (gk, gv) are not provided")
    if beta is None:
        beta = torch.ones_like(q[..., 0])
        if v.shape[2] != q.shape[2]:
            beta = beta.repeat_interleave(v.shape[2] // q.shape[2], dim=2)
    if g is None:
        if use_gate_in_kernel:
            raise ValueError("`g` (raw pre-activation) must be provided when `use_gate_in_kernel=True`.")
        g = torch.zeros(v.shape[:3], device=v.device, dtype=torch.float32)
    return chunk_gated_delta_rule(q, k, v, g, beta, scale=scale, initial_state=initial_state,
                                  output_final_state=output_final_state,
                                  use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel, cu_seqlens=cu_seqlens,
                                  transpose_state_layout=transpose_state_layout,
                                  use_gate_in_kernel=use_gate_in_kernel, A_log=A_log, dt_bias=dt_bias)


fused_recurrent_gdn = fused_recurrent_gated_delta_rule
