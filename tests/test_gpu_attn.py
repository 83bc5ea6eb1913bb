"""GPU parity of causal KATA-SPD attention (forward and backward) against the CPU oracle and the
reference's golden fixtures.  Tolerances (relative L2): 1e-5 for fp32 inputs (fp32-exact CUDA-core
kernels), 1e-2 for bf16 / fp16 inputs (tensor-core kernels)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import kata_oracle as ko
from tests.conftest import attn_case_meta

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 1e-2}


def _pka(algo):
    import linatt_b200.parallel_kata_attn as pka

    pka.ALGO = algo
    return pka


@pytest.fixture(autouse=True)
def _reset_algo():
    yield
    _pka("auto")


def draw(seed, B, T, HQ, H, D, Dv, dtype, qscale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, HQ, D, generator=g) * qscale
    k = torch.randn(B, T, H, D, generator=g)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(B, T, H, Dv, generator=g)
    c = (-torch.nn.functional.softplus(torch.randn(B, T, HQ, generator=g))).cumsum(1)
    do = torch.randn(B, T, HQ, Dv, generator=g)
    q, k, v, do = (x.to(dtype) for x in (q, k, v, do))
    return q, k, v, c, do


def run(pka, q, k, v, do, M, score, c=None, grad=True):
    q, k, v = (x.cuda().requires_grad_(grad) for x in (q, k, v))
    cc = c.cuda().requires_grad_(grad) if c is not None else None
    if cc is not None:
        o = pka.parallel_kata_attn_decay(q, k, v, cc, num_groups=M)
    elif score == "sum":
        o = pka.parallel_kata_attn_sum(q, k, v, num_groups=M)
    else:
        o = pka.parallel_kata_attn(q, k, v, num_groups=M)
    out = {"o": o.detach()}
    if grad:
        o.backward(do.cuda())
        out.update(dq=q.grad, dk=k.grad, dv=v.grad)
        if cc is not None:
            out["dc"] = cc.grad
    torch.cuda.synchronize()
    from linatt_b200 import check_device_status

    check_device_status(q.device)
    return {n: x.float().cpu().numpy() for n, x in out.items()}


def oracle(q, k, v, do, M, score, c=None):
    qn, kn, vn, dn = (x.double().numpy() for x in (q, k, v, do))
    cn = c.double().numpy() if c is not None else None
    o, den = ko.attn_fwd(qn, kn, vn, M, None, score, cn)
    dq, dk, dv, dc = ko.attn_bwd(qn, kn, vn, dn, M, None, score, cn)
    out = dict(o=o, dq=dq, dk=dk, dv=dv)
    if c is not None:
        out["dc"] = dc
    return out


def assert_close(got, ref, tol, names=None):
    for n in names or ref.keys():
        e = ko.rel_l2(got[n], ref[n])
        assert np.isfinite(got[n]).all(), f"{n}: non-finite values"
        assert e < tol, f"{n}: rel-L2 {e:.3e} > {tol:g}"


# --------------------------------------------------------------------------------------------
# golden fixtures (reference outputs): fp32 through the fp32-exact kernels
# --------------------------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["concat_m1", "concat_m2", "concat_m4", "concat_m4_d128", "sum_m2", "sum_m4",
                                  "decay_m2", "decay_m4", "gqa_m2"])
def test_golden_fp32(golden, case):
    rec = golden[case]
    m = attn_case_meta(rec)
    pka = _pka("simt")
    t = {n: torch.from_numpy(rec[n]) for n in ("q", "k", "v", "do")}
    c = torch.from_numpy(rec["c"]) if m["decay"] else None
    got = run(pka, t["q"], t["k"], t["v"], t["do"], m["M"], m["score"], c)
    ref = {n: rec[n] for n in ("o", "dq", "dk", "dv")}
    if m["decay"]:
        ref["dc"] = rec["dc"]
    assert_close(got, ref, 1e-5)


@pytest.mark.parametrize("case", ["concat_m1", "concat_m2", "concat_m4", "concat_m4_d128", "sum_m2", "sum_m4",
                                  "decay_m2", "decay_m4", "gqa_m2"])
def test_golden_bf16_tensor_cores(golden, case):
    rec = golden[case]
    m = attn_case_meta(rec)
    pka = _pka("auto")
    t = {n: torch.from_numpy(rec[n]).bfloat16() for n in ("q", "k", "v", "do")}
    c = torch.from_numpy(rec["c"]) if m["decay"] else None
    got = run(pka, t["q"], t["k"], t["v"], t["do"], m["M"], m["score"], c)
    ref = oracle(t["q"].float(), t["k"].float(), t["v"].float(), t["do"].float(), m["M"], m["score"], c)
    assert_close(got, ref, 1e-2)


# --------------------------------------------------------------------------------------------
# config 1: B=2, T=512, H=4, D=Dv=64, fp32, M in {1,2,4}, plain / decay / offset gate
# --------------------------------------------------------------------------------------------
@pytest.mark.parametrize("M", [1, 2, 4])
@pytest.mark.parametrize("variant", ["plain", "decay", "offset"])
def test_config1_fp32(M, variant):
    pka = _pka("auto")
    q, k, v, c, do = draw(10 + M, 2, 512, 4, 4, 64, 64, torch.float32)
    cc = c if variant == "decay" else None
    if variant == "offset":
        g = torch.Generator().manual_seed(99)
        off = torch.sigmoid(torch.randn(2, 512, 4, generator=g))
        qn, kn = ko.augment_offset(q.numpy(), k.numpy(), off.numpy(), M)
        q, k = torch.from_numpy(qn).float(), torch.from_numpy(kn).float()
    got = run(pka, q, k, v, do, M, "concat", cc)
    ref = oracle(q, k, v, do, M, "concat", cc)
    assert_close(got, ref, 1e-5)


# --------------------------------------------------------------------------------------------
# offset gate at the 200M geometry on the tensor cores: 64-wide heads, M = 4 groups of 16, each
# packed with the offset to 32 (kata/layer.py:268-282) -> q/k 128 wide, v 64 wide
# --------------------------------------------------------------------------------------------
@pytest.mark.parametrize("HQ,H,decay", [(2, 2, False), (4, 2, False), (2, 2, True)])
def test_offset_gate_bf16_tensor_cores(HQ, H, decay):
    from linatt_b200 import _lib

    pka = _pka("auto")
    B, T, M = 2, 300, 4
    q, k, v, c, do = draw(31 + HQ, B, T, HQ, H, 64, 64, torch.float32)
    g = torch.Generator().manual_seed(5)
    off = torch.sigmoid(torch.randn(B, T, HQ, generator=g))
    # the packing appends off_t to each query group and 1 to each key group (per key head: the
    # offset of the head's first query head, as the layer's GQA layout would give it)
    qn, _ = ko.augment_offset(q.numpy(), q.numpy(), off.numpy(), M)
    _, kn = ko.augment_offset(k.numpy(), k.numpy(), off[:, :, ::HQ // H].contiguous().numpy(), M)
    qb, kb, vb, dob = (torch.from_numpy(x).bfloat16() if isinstance(x, np.ndarray) else x.bfloat16()
                       for x in (qn, kn, v, do))
    assert qb.shape[-1] == 128 and vb.shape[-1] == 64
    a = _lib.AttnFwdArgs(dtype=1, B=B, T=T, H=H, HQ=HQ, D=128, Dv=64, M=M, score=0, algo=0, scale=1.0,
                         c=16 if decay else None)
    assert _lib.lib().kata_attn_algo(a) == 1  # the tcgen05 kernels, not the fp32 CUDA-core fallback
    cc = c if decay else None
    got = run(pka, qb, kb, vb, dob, M, "concat", cc)
    ref = oracle(qb.float(), kb.float(), vb.float(), dob.float(), M, "concat", cc)
    assert_close(got, ref, 1e-2)


# --------------------------------------------------------------------------------------------
# bf16 / fp16 tensor-core kernels: shapes, ragged T, GQA, sum, decay
# --------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,T,HQ,H,D,M,score,decay", [
    (1, 1, 1, 1, 64, 4, "concat", False),
    (1, 127, 2, 2, 64, 2, "concat", False),
    (2, 128, 1, 1, 128, 4, "concat", False),
    (1, 129, 2, 2, 128, 1, "concat", False),
    (1, 300, 2, 2, 128, 4, "concat", False),
    (1, 300, 4, 2, 128, 4, "concat", False),
    (1, 257, 2, 2, 128, 2, "sum", False),
    (1, 300, 2, 2, 128, 4, "sum", False),
    (1, 300, 2, 2, 64, 4, "concat", True),
    (1, 300, 4, 2, 128, 2, "concat", True),
    (2, 257, 2, 2, 128, 1, "concat", True),
    (1, 520, 1, 1, 128, 8, "concat", False),
])
def test_half_precision_vs_oracle(dtype, B, T, HQ, H, D, M, score, decay):
    pka = _pka("auto")
    q, k, v, c, do = draw(B * 7 + T + M, B, T, HQ, H, D, D, dtype)
    cc = c if decay else None
    got = run(pka, q, k, v, do, M, score, cc)
    ref = oracle(q.float(), k.float(), v.float(), do.float(), M, score, cc)
    if T == 1:
        # one token attends only to itself: o = v, and dq = dk = 0 exactly (dA = dO.v - <o,dO> = 0),
        # so only o and dv carry a relative error; dq, dk must be tiny in absolute terms
        assert_close(got, ref, TOL[dtype], names=("o", "dv"))
        for n in ("dq", "dk"):
            assert np.abs(got[n]).max() < 1e-2
        return
    assert_close(got, ref, TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decay_non_monotone_c_vs_oracle(dtype):
    """Decay with a cumsum c that rises as well as falls: pairs with c_t - c_s > 0 take the clamp
    exp(min(., 0)) = 1 and contribute nothing to dc (GQA, several query and key tiles)."""
    pka = _pka("auto")
    B, T, HQ, H, D, M = 1, 300, 4, 2, 128, 2
    q, k, v, _, do = draw(41, B, T, HQ, H, D, D, dtype)
    g = torch.Generator().manual_seed(42)
    c = (0.3 * torch.randn(B, T, HQ, generator=g)).cumsum(1)
    got = run(pka, q, k, v, do, M, "concat", c)
    ref = oracle(q.float(), k.float(), v.float(), do.float(), M, "concat", c)
    assert_close(got, ref, TOL[dtype])


def test_tensor_core_forward_writes_every_output():
    """NaN-poisoned outputs through the C ABI: every o/den element must be overwritten."""
    from linatt_b200 import _lib

    q, k, v, _, _ = draw(5, 2, 333, 2, 2, 128, 128, torch.bfloat16)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    o = torch.full((2, 333, 2, 128), float("nan"), device="cuda", dtype=torch.bfloat16)
    den = torch.full((2, 333, 2), float("nan"), device="cuda")
    a = _lib.AttnFwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), den=den.data_ptr(),
                         dtype=1, B=2, T=333, H=2, HQ=2, D=128, Dv=128, M=4, score=0, algo=1,
                         scale=1 / math.sqrt(32))
    _lib.check(_lib.lib().kata_attn_fwd(a, torch.cuda.current_stream().cuda_stream), "fwd")
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and torch.isfinite(den).all()


@pytest.mark.parametrize("B,T", [(0, 64), (2, 0)])
@pytest.mark.parametrize("variant", ["concat", "sum", "decay"])
def test_empty_inputs_give_empty_outputs(B, T, variant):
    """An empty batch or sequence returns empty o and empty gradients, as the reference's empty
    launch grid does; nothing is launched."""
    pka = _pka("auto")
    q = torch.randn(B, T, 2, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, T, 2, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, T, 2, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    if variant == "decay":
        c = torch.zeros(B, T, 2, device="cuda", requires_grad=True)
        o = pka.parallel_kata_attn_decay(q, k, v, c, num_groups=2)
    elif variant == "sum":
        o = pka.parallel_kata_attn_sum(q, k, v, num_groups=4)
    else:
        o = pka.parallel_kata_attn(q, k, v, num_groups=4)
    assert o.shape == (B, T, 2, 128) and o.dtype == torch.bfloat16
    o.sum().backward()
    assert q.grad.shape == q.shape and k.grad.shape == k.shape and v.grad.shape == v.shape
    if variant == "decay":
        assert c.grad.shape == c.shape
    o2, den = pka.parallel_kata_attn_fwd(q.detach(), k.detach(), v.detach(), num_groups=4)
    assert o2.shape == (B, T, 2, 128) and den.shape == (B, T, 2)


# --------------------------------------------------------------------------------------------
# config 3 at full size (B=16, T=4096, H=8, D=Dv=128, M=4, bf16): size-independent properties
# --------------------------------------------------------------------------------------------
def test_config3_full_size_forward():
    pka = _pka("auto")
    B, T, H, D = 16, 4096, 8, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = (torch.randn(B, T, H, D, device="cuda", generator=g) / math.sqrt(D)).bfloat16()
    k = (torch.randn(B, T, H, D, device="cuda", generator=g) / math.sqrt(D)).bfloat16()
    v = (torch.randn(B, T, H, D, device="cuda", generator=g) / math.sqrt(D)).bfloat16()
    o, den = pka.parallel_kata_attn_fwd(q, k, v, num_groups=4)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all() and (den > 0).all()
    # linearity in v (o is A v / den): o(v + v') == o(v) + o(v') within bf16 rounding
    v2 = torch.roll(v, 1, dims=0)
    o2, _ = pka.parallel_kata_attn_fwd(q, k, v2, num_groups=4)
    o12, _ = pka.parallel_kata_attn_fwd(q, k, (v.float() + v2.float()).bfloat16(), num_groups=4)
    assert ko.rel_l2(o12.float().cpu().numpy(), (o.float() + o2.float()).cpu().numpy()) < 1e-2
    # full-T oracle on two (b, h) slices
    for b, h in ((0, 0), (15, 7)):
        qs, ks, vs = (x[b:b + 1, :, h:h + 1].float().cpu().numpy() for x in (q, k, v))
        o_ref, den_ref = ko.attn_fwd(qs, ks, vs, 4)
        assert ko.rel_l2(o[b:b + 1, :, h:h + 1].float().cpu().numpy(), o_ref) < 1e-2
        assert ko.rel_l2(den[b:b + 1, :, h:h + 1].cpu().numpy(), den_ref) < 1e-3


def test_config3_full_size_backward():
    """Config 3 backward at full size: T = 4096 means 32 key tiles per query tile, where the fp32
    TMEM accumulation of dQ / dK over many tiles and the bf16 rounding of P and W could drift.
    Checks linearity in dO over the whole problem and dq / dk / dv on two (b, h) slices against
    the fp64 oracle at full T (about 30 s of CPU per slice)."""
    pka = _pka("auto")
    B, T, H, D, M = 16, 4096, 8, 128, 4
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = ((torch.randn(B, T, H, D, device="cuda", generator=g) / math.sqrt(D)).bfloat16() for _ in range(3))
    do = torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16()
    o, den = pka.parallel_kata_attn_fwd(q, k, v, num_groups=M)
    dq, dk, dv = pka.parallel_kata_attn_bwd(q, k, v, o, den, do, M, None)
    torch.cuda.synchronize()
    for x in (dq, dk, dv):
        assert torch.isfinite(x.float()).all()
    # every gradient is linear in dO: grads(dO + dO') == grads(dO) + grads(dO') within bf16 rounding
    do2 = torch.roll(do, 1, dims=0)
    g2 = pka.parallel_kata_attn_bwd(q, k, v, o, den, do2, M, None)
    g12 = pka.parallel_kata_attn_bwd(q, k, v, o, den, (do.float() + do2.float()).bfloat16(), M, None)
    for name, a, b, c in zip(("dq", "dk", "dv"), (dq, dk, dv), g2, g12):
        e = ko.rel_l2(c.float().cpu().numpy(), (a.float() + b.float()).cpu().numpy())
        assert e < 1e-2, f"{name} not linear in dO: {e:.3e}"
    # full-T oracle on two (b, h) slices
    for b, h in ((0, 0), (15, 7)):
        sl = lambda x: x[b:b + 1, :, h:h + 1].float().cpu().numpy()  # noqa: E731
        rdq, rdk, rdv, _ = ko.attn_bwd(sl(q), sl(k), sl(v), sl(do), M)
        for name, got, ref in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
            e = ko.rel_l2(sl(got), ref)
            assert e < 1e-2, f"slice ({b},{h}) {name}: rel-L2 {e:.3e}"


def test_backward_in_a_fresh_process():
    """The backward runs on the framework's autograd worker thread.  In a fresh process that thread
    may not have a current CUDA context when the library encodes its tensor maps (the buffers it
    gets can come from the allocator's cache, so no runtime call binds one): the library must bind
    the device's context itself.  Run a first forward + backward in a new interpreter."""
    import subprocess
    import sys
    from pathlib import Path

    code = (
        "import torch, linatt_b200.parallel_kata_attn as pka\n"
        "x = [torch.randn(1, 300, 2, 128, device='cuda').bfloat16().requires_grad_(True) for _ in range(3)]\n"
        "o = pka.parallel_kata_attn(*x, num_groups=4)\n"
        "o.backward(torch.randn_like(o))\n"
        "torch.cuda.synchronize()\n"
        "assert all(torch.isfinite(t.grad).all() for t in x)\n"
        "print('FRESH_OK')\n"
    )
    root = Path(__file__).resolve().parent.parent
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "FRESH_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
