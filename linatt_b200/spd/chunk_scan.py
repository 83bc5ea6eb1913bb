"""Normalised sum-score SPD attention forward, head-major -- drop-in for ``kata/spd/chunk_scan.py``.

Same public name and signature as the reference:
  spd_chunk_scan(q, k, v, M, mode, scale=None, C=32, eps=1e-6, warps=4) -> (o, den)   (:295-406)

q, k (B, H, T, D), v (B, H, T, DV) head-major; with kappa(x, y) = sum_{g,h} (scale x_g . y_h)^2 (scale
default 1/E, s = sqrt(scale) on both operands as in :312-319):
    den_t = max(sum_{s<=t} kappa(q_t, k_s), eps),   o_t = sum_{s<=t} kappa(q_t, k_s) v_s / den_t
(the reference's output kernel, :166-177), o in q's dtype and den fp32 (B, H, T).  The reference
builds it from per-chunk feature states and a parallel prefix scan over chunks (forward only, no
autograd); here the numerator and the denominator come from the sum-score attention readout of
``kata_delta_fwd`` (phase 2 with U := v) on the tensor cores, and the clamp and division are one
elementwise pass.  Only ``mode="sum"`` exists, as in the reference; C and warps are accepted and
ignored, and T need not be a multiple of C.
"""

from __future__ import annotations

import torch

from .flash_delta import _fwd_call

__all__ = ["spd_chunk_scan"]


def spd_chunk_scan(q, k, v, M, mode, scale=None, C=32, eps=1e-6, warps=4):
    """Tree-scan-equivalent chunked SPD forward (sum mode): returns (o, den)."""
    if mode != "sum":
        raise ValueError("spd_chunk_scan is implemented for mode='sum' (as in the reference)")
    B, H, T, D = q.shape
    if k.shape != q.shape or v.shape[:3] != (B, H, T):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    tm = lambda x: x.transpose(1, 2).contiguous()  # noqa: E731
    with torch.no_grad():
        _, num, den = _fwd_call(tm(q), tm(k), None, None, M, scale, False, 0.0, phases=2, U=tm(v).float(),
                                want_o=True, want_den=True)
        den = den.clamp_min(eps)
        o = (num / den[..., None]).to(q.dtype)
    return o.transpose(1, 2).contiguous(), den.transpose(1, 2).contiguous()
