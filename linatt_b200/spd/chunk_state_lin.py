"""Linear (no delta) SPD attention numerator, head-major -- drop-in for ``kata/spd/chunk_state_lin.py``.

Same public names and signatures as the reference module:
  spd_state_lin(q, k, v, M, scale=None, C=64, BI=None) -> o          (kata/spd/chunk_state_lin.py:507-510)
  _StateLin                                                            (:432-504)

q, k, v head-major (B, H, T, D / DV); o fp32 (B, H, T, DV) is the raw causal numerator
    o_t = sum_{s<=t} kappa(q_t, k_s) v_s,   kappa(x, y) = sum_{g,h} (scale x_g . y_h)^2,
scale defaulting to 1/E (E = D/M), as the reference applies s = sqrt(scale) to both operands (:442,
:449).  The reference runs an O(T) chunked-state Triton kernel and a two-pass backward; here the
numerator is the sum-score attention readout of ``kata_delta_fwd`` (phase 2, U := v), and the
gradients are the sum-score attention backward ``kata_attn_bwd`` run with den := 1 and o := 0 (so its
centring term <o, dO> vanishes): dA = dO v^T, which is exactly the gradient of the raw numerator.
Both run on the tcgen05 kernels for bf16 / fp16 inputs and the fp32-exact kernels for fp32 inputs.
C and BI (Triton tiling knobs) are accepted and ignored; T need not be a multiple of C.  The
gradients come back in the input dtypes, as the reference's do.
"""

from __future__ import annotations

import torch

from .. import _lib
from .flash_delta import _fwd_call, _scale

__all__ = ["spd_state_lin", "_StateLin"]


def _tm(x):
    return x.transpose(1, 2).contiguous()


def _lin_bwd(q, k, v, do, M, scale):
    """(dq, dk, dv) of o = tril(kappa(q, k)) v for upstream do; time-major tensors."""
    dev = _lib.require_cuda(q, k, v, do)
    B, T, H, D = q.shape
    Dv = v.shape[-1]
    dt = torch.promote_types(torch.promote_types(q.dtype, k.dtype), v.dtype)
    if dt not in _lib.DTYPE:
        raise TypeError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16")
    qc, kc, vc, doc = (x.to(dt).contiguous() for x in (q, k, v, do))
    zero_o = torch.zeros(B, T, H, Dv, device=dev, dtype=dt)
    ones = torch.ones(B, T, H, device=dev, dtype=torch.float32)
    dq = torch.empty(B, T, H, D, device=dev, dtype=dt)
    dk = torch.empty(B, T, H, D, device=dev, dtype=dt)
    dv = torch.empty(B, T, H, Dv, device=dev, dtype=dt)
    if B == 0 or T == 0:
        return dq, dk, dv
    st = _lib.status_word(dev)
    a = _lib.AttnBwdArgs(
        q=qc.data_ptr(), k=kc.data_ptr(), v=vc.data_ptr(), o=zero_o.data_ptr(), den=ones.data_ptr(),
        dout=doc.data_ptr(), c=None, dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), dc=None,
        status=st.data_ptr(), dtype=_lib.DTYPE[dt], B=B, T=T, H=H, HQ=H, D=D, Dv=Dv, M=M, score=_lib.SCORE["sum"],
        algo=_lib.ALGO["auto"], scale=_scale(D, M, scale))
    L = _lib.lib()
    nbytes = L.kata_attn_bwd_workspace_bytes(a)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    with torch.cuda.device(dev):
        _lib.check(L.kata_attn_bwd(a, _lib.stream_handle(dev)), "kata_attn_bwd")
    if _lib.SYNC_CHECK:
        _lib.check_device_status(dev)
    return dq, dk, dv


class _StateLin(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, M, scale, C, BI):
        B, H, T, D = q.shape
        if k.shape != q.shape or v.shape[:3] != (B, H, T):
            raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
        if D % M:
            raise ValueError(f"D={D} not divisible by M={M}")
        qt, kt = _tm(q), _tm(k)
        _, o, _ = _fwd_call(qt, kt, None, None, M, scale, False, 0.0, phases=2, U=_tm(v).float(), want_o=True,
                            want_den=False)
        ctx.save_for_backward(q, k, v)
        ctx.M, ctx.scale = M, scale
        return o.transpose(1, 2).contiguous()

    @staticmethod
    def backward(ctx, do):
        q, k, v = ctx.saved_tensors
        dq, dk, dv = _lin_bwd(_tm(q), _tm(k), _tm(v), _tm(do), ctx.M, ctx.scale)
        hm = lambda x, ref: x.transpose(1, 2).to(ref.dtype).contiguous()  # noqa: E731
        return hm(dq, q), hm(dk, k), hm(dv, v), None, None, None, None


def spd_state_lin(q, k, v, M, scale=None, C=64, BI=None):
    """Linear SPD attention numerator (no delta, no normalisation), differentiable; head-major
    q, k, v (B, H, T, *) -> o fp32 (B, H, T, DV)."""
    return _StateLin.apply(q, k, v, M, scale, C, BI)
