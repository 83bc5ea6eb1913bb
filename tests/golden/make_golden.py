"""Generate the golden fixtures that pin the CPU oracle (and the GPU kernels) to the reference.

Run in a container where the reference checkout is importable (the path is taken from
``LINATT_REFERENCE``; it is never needed at test time):

    LINATT_REFERENCE=/path/to/linatt python tests/golden/make_golden.py

For each seeded case it executes the reference's *own* code on fp32 inputs:
  * forward: the Triton kernels ``parallel_kata_attn_fwd_kernel`` (concat, decay) and
    ``parallel_kata_attn_sum_fwd_kernel`` (sum) under the Triton CPU interpreter
    (``TRITON_INTERPRET=1``), called through ``.fn[grid]`` with ``VARLEN=False`` because the
    reference launcher omits that argument (kata/parallel_kata_attn.py:270-287 vs
    kata/kernels/parallel_kata.py:29), plus ``_kata_decay_ref`` (kata/parallel_kata_attn.py:291)
    in float64 as a second witness;
  * backward: ``parallel_kata_attn_bwd`` (:49) / ``parallel_kata_attn_bwd_sum_torch`` (:579) in
    float64 on the interpreter's o/den, and autograd through ``_kata_decay_ref`` in float64 for
    the decayed form (the reference's production backward, :329-347), which also yields dc;
  * offset gate: ``KataAttention._augment_offset`` (kata/layer.py:268).
Inputs follow the measurement plan's draws: q, k, v ~ N(0,1) (k L2-normalised per head), log-decay
-softplus(N(0,1)) cumsummed, offset gate sigmoid(N(0,1)), dO ~ N(0,1); generator seeded per case.
Arrays are stored as float32 in ``tests/golden/kata_attn_golden.npz``.
"""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"
REF = os.environ.get("LINATT_REFERENCE")
if not REF:
    sys.exit("set LINATT_REFERENCE to the reference checkout")
sys.path.insert(0, REF)

import torch  # noqa: E402

from kata.kernels.parallel_kata import (  # noqa: E402
    parallel_kata_attn_fwd_kernel,
    parallel_kata_attn_sum_fwd_kernel,
)
from kata.parallel_kata_attn import (  # noqa: E402
    _kata_decay_ref,
    parallel_kata_attn_bwd,
    parallel_kata_attn_bwd_sum_torch,
)
from kata.layer import KataAttention  # noqa: E402

OUT = Path(__file__).resolve().parent / "kata_attn_golden.npz"

# (name, B, T, HQ, H, D, Dv, M, score, decay)
CASES = [
    ("concat_m1", 1, 100, 1, 1, 64, 64, 1, "concat", False),
    ("concat_m2", 1, 100, 1, 1, 64, 64, 2, "concat", False),
    ("concat_m4", 2, 100, 1, 1, 64, 64, 4, "concat", False),
    ("concat_m4_d128", 1, 130, 1, 1, 128, 128, 4, "concat", False),
    ("sum_m2", 1, 100, 1, 1, 64, 64, 2, "sum", False),
    ("sum_m4", 1, 100, 1, 1, 64, 64, 4, "sum", False),
    ("decay_m2", 1, 100, 1, 1, 64, 64, 2, "concat", True),
    ("decay_m4", 1, 100, 1, 1, 64, 64, 4, "concat", True),
    ("gqa_m2", 1, 100, 2, 1, 64, 64, 2, "concat", False),
]


def draw(seed, B, T, HQ, H, D, Dv):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, HQ, D, generator=g)
    k = torch.randn(B, T, H, D, generator=g)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(B, T, H, Dv, generator=g)
    ell = -torch.nn.functional.softplus(torch.randn(B, T, HQ, generator=g))
    c = ell.cumsum(1)
    do = torch.randn(B, T, HQ, Dv, generator=g)
    return q, k, v, c, do


def triton_fwd(q, k, v, M, scale, score, c):
    B, T, HQ, D = q.shape
    H = k.shape[2]
    Dv = v.shape[-1]
    o = torch.empty(B, T, HQ, Dv)
    den = torch.empty(B, T, HQ)
    bT = bK = 32
    grid = (1, math.ceil(T / bT), B * HQ)
    if score == "concat":
        parallel_kata_attn_fwd_kernel.fn[grid](
            q, k, v, o, den, c if c is not None else den, scale, T, d_k=D, d_v=Dv, H=H, M=M, HQ=HQ,
            G=HQ // H, bT=bT, bV=Dv, bK=bK, HAS_DECAY=c is not None, VARLEN=False)
    else:
        parallel_kata_attn_sum_fwd_kernel.fn[grid](
            q, k, v, o, den, scale, T, H=H, HQ=HQ, G=HQ // H, d_k=D, d_v=Dv, bV=Dv, M=M, E=D // M, bT=bT, bK=bK)
    return o, den


class _OffsetStub:
    """Carries the three attributes KataAttention._augment_offset reads."""

    def __init__(self, M, E):
        self.spd_num_groups = M
        self._off_E = E
        self._off_Epad = max(16, 1 << E.bit_length())


def main():
    out = {}
    for i, (name, B, T, HQ, H, D, Dv, M, score, decay) in enumerate(CASES):
        q, k, v, c, do = draw(1000 + i, B, T, HQ, H, D, Dv)
        scale = 1.0 / math.sqrt(D // M)
        cc = c if decay else None
        o_tr, den_tr = triton_fwd(q, k, v, M, scale, score, cc)
        q64, k64, v64, do64 = (x.double() for x in (q, k, v, do))
        if score == "concat":
            c_ref = (c if decay else torch.zeros(B, T, HQ)).double()
            kr, vr = k64, v64
            if HQ != H:  # _kata_decay_ref is MHA-only; expand kv heads for the witness
                kr = k64.repeat_interleave(HQ // H, dim=2)
                vr = v64.repeat_interleave(HQ // H, dim=2)
            o_ref = _kata_decay_ref(q64, kr, vr, c_ref, M, scale)
        else:
            o_ref = None
        if decay:
            qd, kd, vd, cd = (x.clone().requires_grad_(True) for x in (q64, k64, v64, c.double()))
            o_ad = _kata_decay_ref(qd, kd, vd, cd, M, scale)
            dq, dk, dv, dc = torch.autograd.grad(o_ad, [qd, kd, vd, cd], do64)
        elif score == "concat":
            dq, dk, dv = parallel_kata_attn_bwd(q64, k64, v64, o_tr.double(), den_tr.double(), do64, M, scale)
            dc = None
        else:
            dq, dk, dv = parallel_kata_attn_bwd_sum_torch(q64, k64, v64, o_tr.double(), den_tr.double(), do64, M,
                                                          scale)
            dc = None
        rec = dict(q=q, k=k, v=v, do=do, o=o_tr, den=den_tr, dq=dq, dk=dk, dv=dv)
        if decay:
            rec["c"] = c
            rec["dc"] = dc
        if o_ref is not None:
            rec["o_ref64"] = o_ref
        for key, val in rec.items():
            out[f"{name}/{key}"] = val.detach().float().numpy()
        out[f"{name}/meta"] = np.array([B, T, HQ, H, D, Dv, M, int(score == "sum"), int(decay)], dtype=np.int64)
        print(f"{name}: done", flush=True)

    # offset gate packing (kata/layer.py:268-282)
    g = torch.Generator().manual_seed(77)
    M, E = 2, 32
    q = torch.randn(1, 20, 2, M * E, generator=g)
    k = torch.randn(1, 20, 2, M * E, generator=g)
    off = torch.sigmoid(torch.randn(1, 20, 2, generator=g))
    qi, ki = KataAttention._augment_offset(_OffsetStub(M, E), q, k, off)
    for key, val in dict(q=q, k=k, off=off, q_in=qi, k_in=ki).items():
        out[f"offset_m2/{key}"] = val.float().numpy()
    out["offset_m2/meta"] = np.array([M, E], dtype=np.int64)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
