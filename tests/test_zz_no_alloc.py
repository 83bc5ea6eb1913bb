"""kata_attn_bwd_noalloc: the backward for callers that cannot allocate device memory.

Such callers (a fixed, pre-reserved device-memory budget that forbids further cudaMalloc, or a
plugin host that hands the kernel only its inputs and outputs) cannot provide the workspace that
kata_attn_bwd needs; this entry point uses the library's own fixed scratch array instead.  The
test calls it through the C ABI twice in a row, on different upstream gradients, and checks each
result against kata_attn_bwd with a caller-allocated workspace.  Both run the same kernels on the
same inputs, and dq, dk and dv are written without atomics, so they must agree bit for bit (a stale
scratch entry would show up here); dc is summed with atomics in a scheduling-dependent order and is
held to the bf16 tolerance the other GPU tests use.  This file sorts last so a run that stops at
the first failure has already run every other test; it also passes on its own in a fresh process.
"""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2


def rel_l2(x, ref):
    x, ref = x.double(), ref.double()
    n = ref.norm()
    return float((x - ref).norm() / n) if n > 0 else float((x - ref).norm())


def _fwd(L, _lib, q, k, v, c, M, scale, stream, score=0):
    B, T, HQ, D = q.shape
    H = k.shape[2]
    o = torch.empty(B, T, HQ, v.shape[-1], device="cuda", dtype=q.dtype)
    den = torch.empty(B, T, HQ, device="cuda")
    a = _lib.AttnFwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), c=_lib.ptr(c), o=o.data_ptr(),
                         den=den.data_ptr(), dtype=1, B=B, T=T, H=H, HQ=HQ, D=D, Dv=v.shape[-1], M=M, score=score,
                         algo=0, scale=scale)
    _lib.check(L.kata_attn_fwd(a, stream), "kata_attn_fwd")
    return o, den


def _bwd_args(_lib, q, k, v, o, den, do, c, M, scale, score=0):
    B, T, HQ, D = q.shape
    H = k.shape[2]
    out = dict(dq=torch.empty_like(q), dk=torch.empty_like(k), dv=torch.empty_like(v))
    if c is not None:
        out["dc"] = torch.empty(B, T, HQ, device="cuda")
    a = _lib.AttnBwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), den=den.data_ptr(),
                         dout=do.data_ptr(), c=_lib.ptr(c), dq=out["dq"].data_ptr(), dk=out["dk"].data_ptr(),
                         dv=out["dv"].data_ptr(), dc=_lib.ptr(out.get("dc")), dtype=1, B=B, T=T, H=H, HQ=HQ, D=D,
                         Dv=v.shape[-1], M=M, score=score, algo=0, scale=scale)
    return a, out


@pytest.mark.parametrize("decay", [False, True])
def test_noalloc_matches_workspace_entry_point_twice(decay):
    from linatt_b200 import _lib

    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    B, T, H, D, M = 2, 300, 2, 128, 4
    scale = 1.0 / math.sqrt(D // M)
    g = torch.Generator(device="cuda").manual_seed(7)
    q, k, v = (torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16() for _ in range(3))
    c = (-torch.nn.functional.softplus(torch.randn(B, T, H, device="cuda", generator=g))).cumsum(1) if decay else None
    o, den = _fwd(L, _lib, q, k, v, c, M, scale, stream)
    for call in range(2):  # two calls in a row, each on a new upstream gradient
        do = torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16()
        a_ref, ref = _bwd_args(_lib, q, k, v, o, den, do, c, M, scale)
        nbytes = L.kata_attn_bwd_workspace_bytes(a_ref)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        a_ref.workspace, a_ref.workspace_bytes = ws.data_ptr(), nbytes
        _lib.check(L.kata_attn_bwd(a_ref, stream), "kata_attn_bwd")
        a_na, got = _bwd_args(_lib, q, k, v, o, den, do, c, M, scale)
        _lib.check(L.kata_attn_bwd_noalloc(a_na, stream), "kata_attn_bwd_noalloc")
        torch.cuda.synchronize()
        for name in ref:
            assert torch.isfinite(got[name].float()).all(), f"call {call}: {name} not finite"
            if name == "dc":
                e = rel_l2(got[name], ref[name])
                assert e < TOL, f"call {call}: {name} rel-L2 {e:.3e}"
            else:
                assert torch.equal(got[name], ref[name]), f"call {call}: {name} differs from kata_attn_bwd"


def test_noalloc_runs_the_gram_form_when_it_fits():
    """AUTO on a sum-score problem with groups of 16 (bf16, Dv = 64): the no-allocation backward
    runs the Gram form when its workspace fits in the array, bit-exact against kata_attn_bwd with
    the full workspace; a problem whose Gram workspace does not fit still runs (the parts form)."""
    from linatt_b200 import _lib

    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(17)
    for B, T, H in ((1, 256, 2), (4, 4096, 4)):  # Gram workspace ~1 MB, then ~76 MB (> 16 MiB)
        D, M = 64, 4
        scale = 1.0 / math.sqrt(D // M)
        q, k, v, do = (torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16() for _ in range(4))
        o, den = _fwd(L, _lib, q, k, v, None, M, scale, stream, score=1)
        a_ref, ref = _bwd_args(_lib, q, k, v, o, den, do, None, M, scale, score=1)
        nbytes = L.kata_attn_bwd_workspace_bytes(a_ref)
        assert (nbytes > 16 << 20) == (T == 4096)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        a_ref.workspace, a_ref.workspace_bytes = ws.data_ptr(), nbytes
        _lib.check(L.kata_attn_bwd(a_ref, stream), "kata_attn_bwd")
        a_na, got = _bwd_args(_lib, q, k, v, o, den, do, None, M, scale, score=1)
        _lib.check(L.kata_attn_bwd_noalloc(a_na, stream), "kata_attn_bwd_noalloc")
        torch.cuda.synchronize()
        for name in ref:
            assert torch.isfinite(got[name].float()).all(), f"T={T}: {name} not finite"
            if T == 256:
                assert torch.equal(got[name], ref[name]), f"T={T}: {name} differs from kata_attn_bwd"
            else:  # parts form against the Gram form: the same function, bf16 rounding apart
                e = rel_l2(got[name], ref[name])
                assert e < TOL, f"T={T}: {name} rel-L2 {e:.3e}"


def test_noalloc_rejects_problems_beyond_its_scratch():
    from linatt_b200 import _lib

    L = _lib.lib()
    # B*T*HQ large enough that the backward scratch exceeds the fixed 16 MiB array
    a = _lib.AttnBwdArgs(q=16, k=16, v=16, o=16, den=16, dout=16, dq=16, dk=16, dv=16, dtype=1, B=64, T=8192, H=8,
                         HQ=8, D=128, Dv=128, M=4, score=0, algo=0, scale=1.0)
    assert L.kata_attn_bwd_workspace_bytes(a) > 16 << 20
    assert L.kata_attn_bwd_noalloc(a, None) == -9
    assert b"16 MiB" in L.kata_strerror(-9)
