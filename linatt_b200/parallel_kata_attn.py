"""Drop-in replacement for ``kata/parallel_kata_attn.py`` backed by sm_100a CUDA kernels.

Same function names, signatures, tensor layouts (time-major ``(B, T, H, D)``), dtypes and
autograd semantics as the reference module; ``bT``, ``bK`` and ``use_triton_bwd`` are accepted
for signature compatibility and ignored (tile shapes are fixed by the kernels).  The computation
goes through the C ABI of ``libkata_b200.so`` (``include/kata_b200.h``):

* forward  -> ``kata_attn_fwd``  (reference: ``parallel_kata_attn_fwd_impl`` :211-288,
  ``parallel_kata_attn_sum_fwd_impl`` :539-576)
* backward -> ``kata_attn_bwd``  (reference: ``parallel_kata_attn_bwd_triton`` :364-529,
  ``parallel_kata_attn_bwd`` :49-146, ``parallel_kata_attn_bwd_sum_torch`` :579-653, and the
  autograd recompute of ``_KataDecayFunction.backward`` :329-347, here a closed-form kernel that
  also returns ``dc``).

Differences from the reference that are deliberate: the backward of every variant (any M, GQA,
sum form, decay) runs on the GPU kernels instead of falling back to materialised T x T torch
code; fp32 inputs take the fp32-exact CUDA-core kernels.
"""

from __future__ import annotations

import math
import warnings

import torch

from . import _lib

__all__ = [
    "parallel_kata_attn",
    "ParallelKataAttnFunction",
    "parallel_kata_attn_fwd_impl",
    "parallel_kata_attn_fwd",
    "parallel_kata_attn_bwd",
    "parallel_kata_attn_bwd_triton",
    "parallel_kata_attn_decay",
    "_KataDecayFunction",
    "_kata_decay_fwd",
    "parallel_kata_attn_sum",
    "ParallelKataAttnSumFunction",
    "parallel_kata_attn_sum_fwd_impl",
    "parallel_kata_attn_bwd_sum_torch",
    "parallel_kata_attn_sum_bwd_triton_M4",
    "parallel_kata_attn_sum_bwd_triton_M2",
]

# Kernel family used by every call of this module ("auto" | "tc" | "simt" | "tc_gram").  Tests and
# the bench switch it to exercise one family explicitly; "auto" is the production setting (it runs
# the sum score with groups of 16 on Gram features, "tc_gram", and everything else as "tc" / "simt").
ALGO = "auto"


def _default_scale(d_k: int, num_groups: int) -> float:
    # reference: scale = 1/sqrt(E), E = d_k // M  (kata/parallel_kata_attn.py:241-244)
    return 1.0 / math.sqrt(d_k // num_groups)


def _common_dtype(*ts: torch.Tensor) -> torch.dtype:
    dt = ts[0].dtype
    for t in ts[1:]:
        dt = torch.promote_types(dt, t.dtype)
    if dt not in _lib.DTYPE:
        raise TypeError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16")
    return dt


_SIMT_WARNED: set = set()


def _warn_if_simt(a, dt) -> None:
    """Warn once per shape class when a 16-bit call leaves the tensor-core envelope: AUTO then runs
    the fp32 CUDA-core kernels, an order of magnitude slower than the tcgen05 path."""
    if dt == torch.float32 or ALGO != "auto":
        return
    if _lib.lib().kata_attn_algo(a) != _lib.ALGO["simt"]:
        return
    key = (a.D, a.Dv, a.M, a.score, bool(a.c))
    if key in _SIMT_WARNED:
        return
    _SIMT_WARNED.add(key)
    warnings.warn(
        f"KATA attention with D={a.D}, Dv={a.Dv}, M={a.M}, score={'sum' if a.score else 'concat'}"
        f"{', decay' if a.c else ''} is outside the tensor-core envelope and runs on the fp32 CUDA-core "
        "kernels (much slower)", RuntimeWarning, stacklevel=4)


def _fwd(q, k, v, num_groups, scale, score, c=None, cu=None):
    """cu: optional (N+1) int32 device offsets of packed documents along T (B = 1)."""
    dev = _lib.require_cuda(q, k, v, c)
    B, T, HQ, d_k = q.shape
    H = k.shape[2]
    d_v = v.shape[-1]
    if k.shape[:2] != (B, T) or v.shape[:2] != (B, T) or k.shape[3] != d_k or v.shape[2] != H:
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if HQ % H != 0:
        raise ValueError("GQA requires HQ multiple of H")
    if d_k % num_groups != 0:
        raise ValueError(f"d_k={d_k} not divisible by M={num_groups}")
    if scale is None:
        scale = _default_scale(d_k, num_groups)
    dt = _common_dtype(q, k, v)
    qc, kc, vc = (x.to(dt).contiguous() for x in (q, k, v))
    o = torch.empty(B, T, HQ, d_v, device=dev, dtype=dt)
    den = torch.empty(B, T, HQ, device=dev, dtype=torch.float32)
    if B == 0 or T == 0:  # empty batch or sequence: nothing to launch (the reference's grid is empty)
        return o.to(v.dtype), den
    cc = None
    if c is not None:
        if c.shape != (B, T, HQ):
            raise ValueError(f"c must be (B,T,HQ)={(B, T, HQ)}, got {tuple(c.shape)}")
        cc = c.float().contiguous()
    st = _lib.status_word(dev)
    a = _lib.AttnFwdArgs(
        q=qc.data_ptr(), k=kc.data_ptr(), v=vc.data_ptr(), c=_lib.ptr(cc), o=o.data_ptr(), den=den.data_ptr(),
        status=st.data_ptr(), dtype=_lib.DTYPE[dt], B=B, T=T, H=H, HQ=HQ, D=d_k, Dv=d_v, M=num_groups,
        score=_lib.SCORE[score], algo=_lib.ALGO[ALGO], scale=float(scale),
        cu_seqlens=_lib.ptr(cu), num_seqs=0 if cu is None else cu.numel() - 1)
    _warn_if_simt(a, dt)
    L = _lib.lib()
    nbytes = L.kata_attn_fwd_workspace_bytes(a)  # Gram features of the sum score, else 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev) if nbytes else None
    a.workspace, a.workspace_bytes = _lib.ptr(ws), nbytes
    with torch.cuda.device(dev):
        _lib.check(L.kata_attn_fwd(a, _lib.stream_handle(dev)), "kata_attn_fwd")
    if _lib.SYNC_CHECK:
        _lib.check_device_status(dev)
    if o.dtype != v.dtype:
        o = o.to(v.dtype)
    return o, den


def _bwd(q, k, v, o, den, do, num_groups, scale, score, c=None, cu=None):
    dev = _lib.require_cuda(q, k, v, o, den, do, c)
    B, T, HQ, d_k = q.shape
    H = k.shape[2]
    d_v = v.shape[-1]
    if scale is None:
        scale = _default_scale(d_k, num_groups)
    dt = _common_dtype(q, k, v)
    qc, kc, vc, oc, doc = (x.to(dt).contiguous() for x in (q, k, v, o, do))
    denc = den.float().contiguous()
    dq = torch.empty(B, T, HQ, d_k, device=dev, dtype=dt)
    dk = torch.empty(B, T, H, d_k, device=dev, dtype=dt)
    dv = torch.empty(B, T, H, d_v, device=dev, dtype=dt)
    cc = c.float().contiguous() if c is not None else None
    dc = torch.empty(B, T, HQ, device=dev, dtype=torch.float32) if c is not None else None
    if B == 0 or T == 0:  # empty batch or sequence: nothing to launch
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dc
    st = _lib.status_word(dev)
    a = _lib.AttnBwdArgs(
        q=qc.data_ptr(), k=kc.data_ptr(), v=vc.data_ptr(), o=oc.data_ptr(), den=denc.data_ptr(),
        dout=doc.data_ptr(), c=_lib.ptr(cc), dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(),
        dc=_lib.ptr(dc), workspace=None, workspace_bytes=0, status=st.data_ptr(), dtype=_lib.DTYPE[dt],
        B=B, T=T, H=H, HQ=HQ, D=d_k, Dv=d_v, M=num_groups, score=_lib.SCORE[score], algo=_lib.ALGO[ALGO],
        scale=float(scale), cu_seqlens=_lib.ptr(cu), num_seqs=0 if cu is None else cu.numel() - 1)
    L = _lib.lib()
    nbytes = L.kata_attn_bwd_workspace_bytes(a)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    a.workspace = ws.data_ptr()
    a.workspace_bytes = nbytes
    with torch.cuda.device(dev):
        _lib.check(L.kata_attn_bwd(a, _lib.stream_handle(dev)), "kata_attn_bwd")
    if _lib.SYNC_CHECK:
        _lib.check_device_status(dev)
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dc


# ------------------------------------------------------------------------------------------------
# concat score (kata_quadratic)
# ------------------------------------------------------------------------------------------------
def parallel_kata_attn_bwd(q, k, v, o, den, do, num_groups, scale, bT=64, bK=64):
    """Backward of the concat-score attention; returns ``(dq, dk, dv)`` in the input dtypes.

    Reference: ``parallel_kata_attn_bwd`` (kata/parallel_kata_attn.py:49-146), same signature.
    """
    dq, dk, dv, _ = _bwd(q, k, v, o, den, do, num_groups, scale, "concat")
    return dq, dk, dv


def parallel_kata_attn_bwd_triton(q, k, v, o, den, do, num_groups, scale, bT=64, bK=64):
    """Reference ``parallel_kata_attn_bwd_triton`` (kata/parallel_kata_attn.py:364): same result,
    computed by the CUDA backward for every M and for GQA."""
    return parallel_kata_attn_bwd(q, k, v, o, den, do, num_groups, scale, bT, bK)


class ParallelKataAttnFunction(torch.autograd.Function):
    """Reference: kata/parallel_kata_attn.py:149-195 (saves q, k, v, o, den)."""

    @staticmethod
    def forward(ctx, q, k, v, num_groups, scale, bT, bK, use_triton_bwd):
        if scale is None:
            scale = _default_scale(q.shape[-1], num_groups)
        o, den = parallel_kata_attn_fwd_impl(q, k, v, num_groups, scale, bT, bK)
        ctx.save_for_backward(q, k, v, o, den)
        ctx.num_groups = num_groups
        ctx.scale = scale
        ctx.bT = bT
        ctx.bK = bK
        ctx.use_triton_bwd = use_triton_bwd
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, den = ctx.saved_tensors
        dq, dk, dv = parallel_kata_attn_bwd(q, k, v, o, den, do, ctx.num_groups, ctx.scale, ctx.bT, ctx.bK)
        return dq, dk, dv, None, None, None, None, None


def parallel_kata_attn(q, k, v, num_groups=4, scale=None, bT=64, bK=64, use_triton_bwd=True):
    """Autograd-wrapped causal KATA-SPD attention, concat score (reference :198-208)."""
    return ParallelKataAttnFunction.apply(q, k, v, num_groups, scale, bT, bK, use_triton_bwd)


def parallel_kata_attn_fwd_impl(q, k, v, num_groups, scale, bT, bK, c=None):
    """Forward (causal); returns ``(o, den)`` with o in v's dtype and den fp32 (B, T, HQ).

    Reference: kata/parallel_kata_attn.py:211-288.  ``c`` is the optional (B, T, HQ) fp32
    cumulative log-decay; the score is then multiplied by exp(min(c_t - c_s, 0)).
    """
    return _fwd(q, k, v, num_groups, scale, "concat", c)


def parallel_kata_attn_fwd(q, k, v, num_groups=4, scale=None, bT=64, bK=64):
    """No-autograd forward used by inference (reference :357-361)."""
    if scale is None:
        scale = _default_scale(q.shape[-1], num_groups)
    return parallel_kata_attn_fwd_impl(q, k, v, num_groups, scale, bT, bK)


# ------------------------------------------------------------------------------------------------
# decay
# ------------------------------------------------------------------------------------------------
def _kata_decay_fwd(q, k, v, c, num_groups, scale):
    """Forward of the decayed form returning only o (the reference's ``_kata_decay_ref`` computes
    the same quantity by materialising T x T, kata/parallel_kata_attn.py:291-310)."""
    if scale is None:
        scale = _default_scale(q.shape[-1], num_groups)
    o, _ = _fwd(q, k, v, num_groups, scale, "concat", c)
    return o


class _KataDecayFunction(torch.autograd.Function):
    """Reference: kata/parallel_kata_attn.py:313-347.  The reference recomputes the T x T torch
    graph in fp32 for its backward; here the backward is the CUDA kernel with closed-form dc."""

    @staticmethod
    def forward(ctx, q, k, v, c, num_groups, scale):
        if scale is None:
            scale = _default_scale(q.shape[-1], num_groups)
        o, den = _fwd(q, k, v, num_groups, scale, "concat", c)
        ctx.save_for_backward(q, k, v, c, o, den)
        ctx.num_groups, ctx.scale = num_groups, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, c, o, den = ctx.saved_tensors
        dq, dk, dv, dc = _bwd(q, k, v, o, den, do, ctx.num_groups, ctx.scale, "concat", c)
        return dq, dk, dv, dc.to(c.dtype), None, None


def parallel_kata_attn_decay(q, k, v, c, num_groups=2, scale=None):
    """Decayed SPD attention o_t = sum_{s<=t} exp(c_t-c_s)(q.k)^2 v_s / sum(...) (reference :350-354)."""
    return _KataDecayFunction.apply(q, k, v, c, num_groups, scale)


# ------------------------------------------------------------------------------------------------
# sum score (kata_quadratic_sum)
# ------------------------------------------------------------------------------------------------
def parallel_kata_attn_sum_fwd_impl(q, k, v, num_groups, scale, bT, bK):
    """Sum-SPD forward, A = sum_{i,j} (scale q_i.k_j)^2; returns (o, den) (reference :539-576)."""
    if scale is None:
        scale = _default_scale(q.shape[-1], num_groups)
    return _fwd(q, k, v, num_groups, scale, "sum")


def parallel_kata_attn_bwd_sum_torch(q, k, v, o, den, do, num_groups, scale):
    """Sum-SPD backward with the reference's signature (kata/parallel_kata_attn.py:579-653),
    computed by the CUDA kernel for every M and for GQA."""
    dq, dk, dv, _ = _bwd(q, k, v, o, den, do, num_groups, scale, "sum")
    return dq, dk, dv


def parallel_kata_attn_sum_bwd_triton_M4(q, k, v, o, den, do, scale):
    """Reference :755-827 (M=4, MHA)."""
    return parallel_kata_attn_bwd_sum_torch(q, k, v, o, den, do, 4, scale)


def parallel_kata_attn_sum_bwd_triton_M2(q, k, v, o, den, do, scale):
    """Reference :830-901 (M=2)."""
    return parallel_kata_attn_bwd_sum_torch(q, k, v, o, den, do, 2, scale)


class ParallelKataAttnSumFunction(torch.autograd.Function):
    """Reference: kata/parallel_kata_attn.py:656-734 (saves q, k, v, o, den)."""

    @staticmethod
    def forward(ctx, q, k, v, num_groups, scale, bT, bK, use_triton_bwd):
        if scale is None:
            scale = _default_scale(q.shape[-1], num_groups)
        o, den = parallel_kata_attn_sum_fwd_impl(q, k, v, num_groups, scale, bT, bK)
        ctx.save_for_backward(q, k, v, o, den)
        ctx.num_groups = num_groups
        ctx.scale = scale
        ctx.use_triton_bwd = use_triton_bwd
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, den = ctx.saved_tensors
        dq, dk, dv = parallel_kata_attn_bwd_sum_torch(q, k, v, o, den, do, ctx.num_groups, ctx.scale)
        return dq, dk, dv, None, None, None, None, None


def parallel_kata_attn_sum(q, k, v, num_groups=4, scale=None, bT=64, bK=64, use_triton_bwd=True):
    """Autograd-wrapped sum-SPD causal attention (reference :737-752)."""
    return ParallelKataAttnSumFunction.apply(q, k, v, num_groups, scale, bT, bK, use_triton_bwd)
