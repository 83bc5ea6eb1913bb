"""SPD delta rule (DeltaKATA) -- drop-in for ``kata/spd/flash_delta.py``.

Same public names and signatures as the reference module:
  flash_delta(q, k, v, beta, M, scale=None, C=64, normalize=False, eps=1e-5) -> o      (:1111-1116)
  _FlashDelta                                                                          (:1060-1108)
  flash_delta_U(q, k, v, beta, M, scale=None, C=64, warps=4) -> U                      (:186-212)
  flash_delta_readout(q, k, U, M, scale=None, C=64, BM=128) -> o                       (:975-983)
  flash_delta_den(q, k, M, scale=None, C=64, BM=128) -> den                            (:1049-1057)
  flash_delta_bwd(q, k, v, beta, U, do, M, scale=None, C=64, z=None) -> dq,dk,dv,dbeta (:830-895)

Math (time-major (B,T,H,D) inputs; kappa(x,y) = sum_{g,h} (scale x_g . y_h)^2, scale default 1/E):
  U = (I + diag(beta) tril(kappa(k,k),-1))^{-1} diag(beta) v,  o = tril(kappa(q,k)) U
  normalize: den_t = sum_{s<=t} kappa(q_t,k_s), o = num/(den+eps), with the reference's consistent
  backward (dO' = dO/den, dA_qk centred by z_t = <dO_t,o_t>/den_t).
All compute runs in ``libkata_b200.so`` (``kata_delta_fwd`` / ``kata_delta_bwd``): the kernel value
is the attention "sum" score, so the readout and every O(T^2) gradient product run on the attention
kernels (tcgen05 tensor cores for bf16 / fp16 inputs, fp32-exact CUDA cores for fp32 inputs), and
the triangular solves for U and its adjoint run as O(T) chunk scans over the E^2-feature state.
Differences from the reference: T need not be a multiple of C (C, warps and BM are accepted and
ignored); o and the gradients come out fp32 and are cast to the input dtypes exactly as the
reference does.
"""

from __future__ import annotations

import torch

from .. import _lib

__all__ = [
    "flash_delta",
    "flash_delta_U",
    "flash_delta_readout",
    "flash_delta_den",
    "flash_delta_bwd",
]


def _scale(D: int, M: int, scale):
    # reference: s = (1/E if scale is None else scale) ** 0.5 applied to both operands (:193, :202)
    return 1.0 / (D // M) if scale is None else float(scale)


def _qkv_dtype(*ts):
    dt = ts[0].dtype
    for t in ts[1:]:
        if t is not None:
            dt = torch.promote_types(dt, t.dtype)
    if dt not in _lib.DTYPE:
        raise TypeError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16")
    return dt


def _prep(dt, *ts):
    return [None if t is None else t.to(dt).contiguous() for t in ts]


def _fwd_call(q, k, v, beta, M, scale, normalize, eps, phases, U=None, want_o=True, want_den=True, want_E=False,
              state=None):
    dev = _lib.require_cuda(q, k, v, beta, U)
    B, T, H, D = q.shape
    if k.shape != q.shape:
        raise ValueError(f"k shape {tuple(k.shape)} != q shape {tuple(q.shape)}")
    Dv = v.shape[-1] if v is not None else (U.shape[-1] if U is not None else D)
    dt = _qkv_dtype(q, k, v)
    qc, kc, vc = _prep(dt, q, k, v)
    bc = None if beta is None else beta.float().contiguous()
    f32 = dict(device=dev, dtype=torch.float32)
    if phases != 2:
        U = torch.empty(B, T, H, Dv, **f32)
    else:
        U = None if U is None else U.float().contiguous()
    o = torch.empty(B, T, H, Dv, **f32) if want_o else None
    den = torch.empty(B, T, H, **f32) if want_den else None
    E = torch.empty(B, T, H, Dv, **f32) if want_E else None
    a = _lib.DeltaFwdArgs(
        q=qc.data_ptr(), k=kc.data_ptr(), v=_lib.ptr(vc), beta=_lib.ptr(bc), U=_lib.ptr(U), E=_lib.ptr(E),
        o=_lib.ptr(o), den=_lib.ptr(den), dtype=_lib.DTYPE[dt], B=B, T=T, H=H, D=D, Dv=Dv, M=M,
        normalize=int(bool(normalize)), scale=_scale(D, M, scale), eps=float(eps), phases=phases,
        state=_lib.ptr(state))
    L = _lib.lib()
    ws = torch.empty(int(L.kata_delta_fwd_workspace_bytes(a)), device=dev, dtype=torch.uint8)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(dev):
        _lib.check(L.kata_delta_fwd(a, _lib.stream_handle(dev)), "kata_delta_fwd")
    return (U, o, den, E) if want_E else (U, o, den)


def _bwd_call(q, k, v, beta, U, do, M, scale, normalize, eps, o=None, den=None, z=None, E=None):
    dev = _lib.require_cuda(q, k, v, beta, U, do, o, den, z, E)
    B, T, H, D = q.shape
    Dv = v.shape[-1]
    dt = _qkv_dtype(q, k, v)
    qc, kc, vc = _prep(dt, q, k, v)
    bc, Uc, doc, oc, denc, zc, Ec = _prep(torch.float32, beta, U, do, o, den, z, E)
    f32 = dict(device=dev, dtype=torch.float32)
    dq = torch.empty(B, T, H, D, **f32)
    dk = torch.empty(B, T, H, D, **f32)
    dv = torch.empty(B, T, H, Dv, **f32)
    dbeta = torch.empty(B, T, H, **f32)
    a = _lib.DeltaBwdArgs(
        q=qc.data_ptr(), k=kc.data_ptr(), v=vc.data_ptr(), beta=bc.data_ptr(), U=Uc.data_ptr(), E=_lib.ptr(Ec),
        o=_lib.ptr(oc), den=_lib.ptr(denc), dout=doc.data_ptr(), z=_lib.ptr(zc), dq=dq.data_ptr(),
        dk=dk.data_ptr(), dv=dv.data_ptr(), dbeta=dbeta.data_ptr(), workspace=None, workspace_bytes=0,
        dtype=_lib.DTYPE[dt], B=B, T=T, H=H, D=D, Dv=Dv, M=M, normalize=int(bool(normalize)),
        scale=_scale(D, M, scale), eps=float(eps))
    L = _lib.lib()
    ws = torch.empty(int(L.kata_delta_bwd_workspace_bytes(a)), device=dev, dtype=torch.uint8)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    with torch.cuda.device(dev):
        _lib.check(L.kata_delta_bwd(a, _lib.stream_handle(dev)), "kata_delta_bwd")
    return dq, dk, dv, dbeta


def flash_delta_U(q, k, v, beta, M, scale=None, C=64, warps=4):
    """U = (I + diag(beta) tril(A_kk,-1))^{-1} diag(beta) v, fp32 (B,T,H,Dv)."""
    U, _, _ = _fwd_call(q, k, v, beta, M, scale, False, 0.0, phases=1, want_o=False, want_den=False)
    return U


def flash_delta_readout(q, k, U, M, scale=None, C=64, BM=128):
    """numerator tril(A_qk) U, fp32 (B,T,H,Dv)."""
    _, o, _ = _fwd_call(q, k, None, None, M, scale, False, 0.0, phases=2, U=U, want_o=True, want_den=False)
    return o


def flash_delta_den(q, k, M, scale=None, C=64, BM=128):
    """den_t = sum_{s<=t} A_qk[t,s], fp32 (B,T,H)."""
    _, _, den = _fwd_call(q, k, None, None, M, scale, False, 0.0, phases=2, want_o=False, want_den=True)
    return den


def flash_delta_bwd(q, k, v, beta, U, do, M, scale=None, C=64, z=None):
    """(dq, dk, dv, dbeta) fp32 for the raw numerator given dO' = ``do`` and centring ``z``
    (z=None -> 0), the reference's contract (:830-895)."""
    if z is None:
        B, T, H, _ = q.shape
        z = torch.zeros(B, T, H, device=q.device, dtype=torch.float32)
    return _bwd_call(q, k, v, beta, U, do, M, scale, False, 0.0, z=z)


class _FlashDelta(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, beta, M, scale, C, normalize, eps):
        U, o, den, E = _fwd_call(q, k, v, beta, M, scale, normalize, eps, phases=0, want_E=True)
        # Besides the reference's saved set (q, k, v, beta, U [, den, o]) the erase term E is kept so
        # that the backward does not repeat the forward scan.
        if normalize:
            ctx.save_for_backward(q, k, v, beta, U, den, o, E)
        else:
            ctx.save_for_backward(q, k, v, beta, U, E)
        ctx.M, ctx.scale, ctx.C, ctx.normalize, ctx.eps = M, scale, C, normalize, eps
        return o

    @staticmethod
    def backward(ctx, do):
        if ctx.normalize:
            q, k, v, beta, U, den, o, E = ctx.saved_tensors
            dq, dk, dv, db = _bwd_call(q, k, v, beta, U, do, ctx.M, ctx.scale, True, ctx.eps, o=o, den=den, E=E)
        else:
            q, k, v, beta, U, E = ctx.saved_tensors
            B, T, H, _ = q.shape
            z = torch.zeros(B, T, H, device=q.device, dtype=torch.float32)
            dq, dk, dv, db = _bwd_call(q, k, v, beta, U, do, ctx.M, ctx.scale, False, 0.0, z=z, E=E)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), db.to(beta.dtype), None, None, None, None, None


def flash_delta(q, k, v, beta, M, scale=None, C=64, normalize=False, eps=1e-5):
    """Trainable full-SPD delta rule; o is fp32 (B,T,H,Dv).  normalize=True -> o = num/(den+eps)."""
    return _FlashDelta.apply(q, k, v, beta, M, scale, C, normalize, eps)
