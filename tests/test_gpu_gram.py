"""GPU parity of the sum score on Gram features (KATA_ALGO_TC_GRAM: groups of 16, bf16, Dv = 64).

The sum score scale^2 sum_{a,b} (q_a . k_b)^2 equals <phi(q), phi(k)> over the 136 entries of the
group Gram matrix; the library runs it as a linear score on the tensor cores.  Checked here against
the fp64 oracle (which squares the M^2 parts, as the reference does), against the parts-form
tensor-core kernels on the same inputs, and through the entry-point variants: the split dq / dk-dv
passes, q and k given as one tensor (the delta rule's erase-term backward), GQA, ragged T and
D = 128 with M = 8 (no parts-form tensor-core kernel exists there).  Tolerance: rel-L2 1e-2, the
bf16 bar of the other tensor-core tests; variants of one computation must agree bit for bit.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from tests.test_gpu_attn import _pka, assert_close, draw, oracle, run

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _reset_algo():
    yield
    _pka("auto")


@pytest.mark.parametrize("B,T,HQ,H,D,M", [
    (1, 1, 1, 1, 64, 4),
    (1, 127, 2, 2, 64, 4),
    (2, 300, 2, 2, 64, 4),
    (1, 520, 4, 2, 64, 4),
    (1, 300, 2, 2, 128, 8),
    (1, 257, 2, 1, 128, 8),
])
def test_gram_vs_oracle(B, T, HQ, H, D, M):
    from linatt_b200 import _lib

    a = _lib.AttnFwdArgs(dtype=1, B=B, T=T, H=H, HQ=HQ, D=D, Dv=64, M=M, score=1, algo=0, scale=1.0)
    assert _lib.lib().kata_attn_algo(a) == 3  # AUTO takes the Gram form here
    pka = _pka("tc_gram")
    q, k, v, _, do = draw(B * 11 + T + M, B, T, HQ, H, D, 64, torch.bfloat16)
    got = run(pka, q, k, v, do, M, "sum")
    ref = oracle(q.float(), k.float(), v.float(), do.float(), M, "sum")
    if T == 1:  # o = v and dq = dk = 0 exactly (see test_half_precision_vs_oracle)
        assert_close(got, ref, 1e-2, names=("o", "dv"))
        for n in ("dq", "dk"):
            assert np.abs(got[n]).max() < 1e-2
        return
    assert_close(got, ref, 1e-2)


def test_gram_matches_parts_form_at_the_delta_geometry():
    """The delta rule's attention geometry (D = Dv = 64, M = 4, sum score): the Gram form against the
    parts form (AUTO before the Gram form existed) and both against the oracle."""
    B, T, H, D, M = 2, 1024, 3, 64, 4
    q, k, v, _, do = draw(404, B, T, H, H, D, D, torch.bfloat16)
    gram = run(_pka("tc_gram"), q, k, v, do, M, "sum")
    parts = run(_pka("tc"), q, k, v, do, M, "sum")
    ref = oracle(q.float(), k.float(), v.float(), do.float(), M, "sum")
    assert_close(gram, ref, 1e-2)
    assert_close(parts, ref, 1e-2)
    assert_close(gram, parts, 1e-2)


def _fwd_bwd_capi(q, k, v, do, M, *, phases_split=False, algo=3):
    """kata_attn_fwd + kata_attn_bwd through the C ABI (sum score), the backward either whole or as
    the dq pass followed by the dk/dv pass on the same workspace."""
    from linatt_b200 import _lib

    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    B, T, HQ, D = q.shape
    H, Dv = k.shape[2], v.shape[-1]
    scale = 1.0 / math.sqrt(D // M)
    o = torch.empty(B, T, HQ, Dv, device="cuda", dtype=q.dtype)
    den = torch.empty(B, T, HQ, device="cuda")
    fa = _lib.AttnFwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), den=den.data_ptr(),
                          dtype=1, B=B, T=T, H=H, HQ=HQ, D=D, Dv=Dv, M=M, score=1, algo=algo, scale=scale)
    nf = L.kata_attn_fwd_workspace_bytes(fa)
    wf = torch.empty(max(nf, 1), dtype=torch.uint8, device="cuda")
    fa.workspace, fa.workspace_bytes = wf.data_ptr(), nf
    _lib.check(L.kata_attn_fwd(fa, stream), "kata_attn_fwd")
    out = dict(o=o, den=den, dq=torch.empty_like(q), dk=torch.empty_like(k), dv=torch.empty_like(v))
    ba = _lib.AttnBwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), den=den.data_ptr(),
                          dout=do.data_ptr(), dq=out["dq"].data_ptr(), dk=out["dk"].data_ptr(), dv=out["dv"].data_ptr(),
                          dtype=1, B=B, T=T, H=H, HQ=HQ, D=D, Dv=Dv, M=M, score=1, algo=algo, scale=scale)
    nb = L.kata_attn_bwd_workspace_bytes(ba)
    wb = torch.empty(nb, dtype=torch.uint8, device="cuda")
    ba.workspace, ba.workspace_bytes = wb.data_ptr(), nb
    for ph in ((1, 2) if phases_split else (0,)):
        ba.phases = ph
        _lib.check(L.kata_attn_bwd(ba, stream), "kata_attn_bwd")
    torch.cuda.synchronize()
    _lib.check_device_status(q.device)
    return out


def test_gram_split_passes_and_shared_qk_tensor_are_bit_exact():
    B, T, H, D, M = 2, 384, 2, 64, 4
    g = torch.Generator(device="cuda").manual_seed(21)
    k, v, do = (torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16() for _ in range(3))
    k = (k.float() / k.float().norm(dim=-1, keepdim=True)).bfloat16()
    whole = _fwd_bwd_capi(k, k, v, do, M)                        # q and k: one tensor, one feature map
    split = _fwd_bwd_capi(k, k, v, do, M, phases_split=True)     # dq pass, then dk/dv pass
    copy = _fwd_bwd_capi(k.clone(), k, v, do, M)                 # q a separate copy of k
    for name in whole:
        assert torch.isfinite(whole[name].float()).all(), name
        assert torch.equal(whole[name], split[name]), f"{name}: split passes differ"
        assert torch.equal(whole[name], copy[name]), f"{name}: shared q/k tensor differs from a copy"
