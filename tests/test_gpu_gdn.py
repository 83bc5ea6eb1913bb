"""GPU parity of the gated delta rule (``linatt_b200.gated_delta_rule.chunk_gated_delta_rule``, the
drop-in for fla's entry point) against fla's own naive references (golden fixtures) and the fp64
oracle.  Tolerances (relative L2): 1e-5 for fp32 inputs, 1e-2 for bf16 inputs (oracle run on the
same bf16-rounded values)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import gdn_oracle as go
from oracle.kata_oracle import rel_l2

pytestmark = pytest.mark.gpu

GRADS = ("dq", "dk", "dv", "dg", "dbeta")


def _golden():
    from tests.conftest import GOLDEN

    z = np.load(GOLDEN / "gdn_golden.npz")
    out = {}
    for key in z.files:
        case, name = key.split("/")
        out.setdefault(case, {})[name] = z[key]
    return out


def run(q, k, v, g, beta, do, h0=None, dht=None, cu=None, **kw):
    from linatt_b200.gated_delta_rule import chunk_gated_delta_rule

    leaves = [x.cuda().requires_grad_(True) for x in (q, k, v, g, beta)]
    h0c = h0.cuda().requires_grad_(True) if h0 is not None else None
    extra = {}
    for name in ("A_log", "dt_bias"):
        if name in kw:
            extra[name] = kw.pop(name).cuda().requires_grad_(True)
    o, ht = chunk_gated_delta_rule(*leaves, initial_state=h0c, output_final_state=True,
                                   cu_seqlens=None if cu is None else cu.cuda(), **kw, **extra)
    loss = (o.float() * do.cuda().float()).sum()
    if dht is not None:
        loss = loss + (ht * dht.cuda()).sum()
    loss.backward()
    out = {"o": o.detach(), "ht": ht.detach()}
    for n, x in zip(GRADS, leaves):
        out[n] = x.grad
    if h0c is not None:
        out["dh0"] = h0c.grad
    for n, x in extra.items():
        out["d" + n] = x.grad
    return out


def np64(x):
    return x.detach().cpu().double().numpy()


@pytest.mark.parametrize("case", ["basic", "chunk_t128", "varlen"])
def test_gdn_fp32_matches_fla_naive_golden(case):
    rec = _golden()[case]
    t = lambda n: torch.from_numpy(rec[n]).float()
    h0 = t("h0") if "h0" in rec else None
    cu = torch.from_numpy(rec["cu_seqlens"]) if "cu_seqlens" in rec else None
    got = run(t("q"), t("k"), t("v"), t("g"), t("beta"), t("do"), h0=h0, dht=t("dht"), cu=cu)
    assert rel_l2(np64(got["o"]), rec["o"]) < 1e-5
    assert rel_l2(np64(got["ht"]), rec["ht"]) < 1e-5
    for n in GRADS + (("dh0",) if h0 is not None else ()):
        e = rel_l2(np64(got[n]), rec[n])
        assert e < 1e-5, f"{n}: rel-L2 {e:.3e}"


def draw(seed, B, T, H, HV, K, V, dtype=torch.float32, h0=False):
    g_ = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=g_)
    k = F.normalize(torch.randn(B, T, H, K, generator=g_), dim=-1)
    v = torch.randn(B, T, HV, V, generator=g_)
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=g_))
    g = -F.softplus(torch.randn(B, T, HV, generator=g_))
    do = torch.randn(B, T, HV, V, generator=g_)
    s0 = torch.randn(B, HV, K, V, generator=g_) * 0.1 if h0 else None
    dht = torch.randn(B, HV, K, V, generator=g_) * 0.1
    q, k, v = (x.to(dtype) for x in (q, k, v))
    return q, k, v, g, beta, do, s0, dht


def oracle(q, k, v, g, beta, do, h0=None, dht=None, cu=None, **kw):
    f = lambda x: None if x is None else x.double().numpy()
    kw = {n: (f(x) if isinstance(x, torch.Tensor) else x) for n, x in kw.items()}
    return go.gdn(f(q), f(k), f(v), f(g), f(beta), initial_state=f(h0), output_final_state=True,
                  cu_seqlens=None if cu is None else cu.numpy(), grad_out=f(do), grad_final=f(dht), **kw)


@pytest.mark.parametrize("B,T,H,HV,K,V,h0", [(2, 200, 2, 4, 64, 64, True), (1, 64, 1, 1, 64, 64, False),
                                             (1, 1, 1, 1, 64, 64, True), (3, 130, 2, 2, 48, 40, True)])
def test_gdn_fp32_matches_oracle(B, T, H, HV, K, V, h0):
    q, k, v, g, beta, do, s0, dht = draw(T + HV, B, T, H, HV, K, V, h0=h0)
    got = run(q, k, v, g, beta, do, h0=s0, dht=dht)
    ref = oracle(q, k, v, g, beta, do, h0=s0, dht=dht)
    assert rel_l2(np64(got["o"]), ref["o"]) < 1e-5
    assert rel_l2(np64(got["ht"]), ref["final_state"]) < 1e-5
    for n in GRADS + (("dh0",) if h0 else ()):
        e = rel_l2(np64(got[n]), ref[n])
        assert e < 1e-5, f"{n}: rel-L2 {e:.3e}"


@pytest.mark.parametrize("dtype,V,HV,h0", [(torch.float32, 128, 2, True), (torch.float32, 96, 4, True),
                                            (torch.bfloat16, 128, 2, False)])
def test_gdn_value_heads_wider_than_the_kernels(dtype, V, HV, h0):
    """V > 64: the state's value columns evolve independently, so the value head runs as 64-column
    slices whose q, k, g, beta gradients add up; the result equals the fp64 oracle on the whole head."""
    B, T, H, K = 2, 150, 2, 64
    q, k, v, g, beta, do, s0, dht = draw(V + HV, B, T, H, HV, K, V, h0=h0, dtype=dtype)
    got = run(q, k, v, g, beta, do, h0=s0, dht=dht)
    ref = oracle(q, k, v, g, beta, do, h0=s0, dht=dht)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert got["o"].shape[-1] == V and got["ht"].shape[-1] == V
    assert rel_l2(np64(got["o"]), ref["o"]) < tol
    assert rel_l2(np64(got["ht"]), ref["final_state"]) < tol
    for n in GRADS + (("dh0",) if h0 else ()):
        e = rel_l2(np64(got[n]), ref[n])
        assert e < tol, f"{n}: rel-L2 {e:.3e}"


def test_gdn_gate_l2norm_transpose_options():
    B, T, H, HV, K, V = 1, 150, 2, 2, 64, 64
    q, k, v, g, beta, do, s0, dht = draw(4, B, T, H, HV, K, V, h0=True)
    A_log = torch.randn(HV) * 0.3
    dt_bias = torch.randn(HV) * 0.3
    kw = dict(use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=A_log, dt_bias=dt_bias)
    got = run(q, k, v, g, beta, do, h0=s0, dht=dht, **dict(kw))
    ref = oracle(q, k, v, g, beta, do, h0=s0, dht=dht, **kw)
    for n, r in (("o", "o"), ("ht", "final_state")):
        assert rel_l2(np64(got[n]), ref[r]) < 1e-5, n
    for n in GRADS + ("dh0", "dA_log", "ddt_bias"):
        e = rel_l2(np64(got[n]), ref[n])
        assert e < 1e-5, f"{n}: rel-L2 {e:.3e}"
    # transposed state layout: h0 / ht / dh0 as (N, HV, V, K)
    from linatt_b200.gated_delta_rule import chunk_gated_delta_rule

    h0t = s0.transpose(-1, -2).contiguous().cuda().requires_grad_(True)
    o, ht = chunk_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), initial_state=h0t,
                                   output_final_state=True, transpose_state_layout=True)
    ref0 = oracle(q, k, v, g, beta, do, h0=s0, dht=dht)
    assert rel_l2(np64(ht.transpose(-1, -2)), ref0["final_state"]) < 1e-5
    ((o * do.cuda()).sum() + (ht * dht.transpose(-1, -2).cuda()).sum()).backward()
    assert rel_l2(np64(h0t.grad.transpose(-1, -2)), ref0["dh0"]) < 1e-5


def test_gdn_varlen_matches_oracle():
    cu = torch.tensor([0, 1, 65, 200, 333], dtype=torch.int64)
    T = int(cu[-1])
    q, k, v, g, beta, do, _, _ = draw(8, 1, T, 2, 2, 64, 64)
    g_ = torch.Generator().manual_seed(9)
    s0 = torch.randn(4, 2, 64, 64, generator=g_) * 0.1
    dht = torch.randn(4, 2, 64, 64, generator=g_) * 0.1
    got = run(q, k, v, g, beta, do, h0=s0, dht=dht, cu=cu)
    ref = oracle(q, k, v, g, beta, do, h0=s0, dht=dht, cu=cu)
    assert rel_l2(np64(got["o"]), ref["o"]) < 1e-5
    assert rel_l2(np64(got["ht"]), ref["final_state"]) < 1e-5
    for n in GRADS + ("dh0",):
        e = rel_l2(np64(got[n]), ref[n])
        assert e < 1e-5, f"{n}: rel-L2 {e:.3e}"


def test_gdn_bf16_config2_full_size():
    """Config 2 (B8 T2048 H12 K=V=64, bf16) against the fp64 oracle on the same bf16 inputs."""
    B, T, H, K, V = 8, 2048, 12, 64, 64
    q, k, v, g, beta, do, _, _ = draw(0, B, T, H, H, K, V, dtype=torch.bfloat16)
    got = run(q, k, v, g, beta, do)
    assert got["dq"].dtype == torch.bfloat16 and got["o"].dtype == torch.bfloat16
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = oracle(q, k, v, g, beta, do)
    assert rel_l2(np64(got["o"]), ref["o"]) < 1e-2
    for n in GRADS:
        e = rel_l2(np64(got[n]), ref[n])
        assert e < 1e-2, f"{n}: rel-L2 {e:.3e}"


def test_gdn_backward_recompute_path_matches_reuse():
    """The C ABI's backward without the forward workspace (recomputing the chunk states from the
    saved A) gives the same gradients as the autograd path, which passes the forward workspace."""
    from linatt_b200 import gated_delta_rule as gdr

    B, T, H, K, V = 2, 300, 2, 64, 64
    q, k, v, g, beta, do, s0, dht = draw(12, B, T, H, H, K, V, h0=True)
    qc, kc, vc, gc, bc, s0c, doc, dhtc = (x.cuda().contiguous() for x in (q, k, v, g, beta, s0, do, dht))
    tables = gdr._chunk_tables(None, None, B, T, qc.device)
    o, A, ht, ws = gdr._fwd(qc, kc, vc, gc, bc, K ** -0.5, s0c, True, tables)
    a = gdr._bwd(qc, kc, vc, gc, bc, A, K ** -0.5, s0c, doc, dhtc, tables, fwd_ws=ws)
    b = gdr._bwd(qc, kc, vc, gc, bc, A, K ** -0.5, s0c, doc, dhtc, tables, fwd_ws=None)
    for x, y in zip(a, b):
        assert rel_l2(np64(x), np64(y)) < 1e-6


def test_fused_recurrent_entry_point_matches_oracle():
    from linatt_b200.gated_delta_rule import fused_recurrent_gated_delta_rule

    B, T, H, K, V = 2, 40, 2, 64, 64
    q, k, v, g, beta, do, s0, dht = draw(21, B, T, H, H, K, V, h0=True)
    o, ht = fused_recurrent_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g=g.cuda(), beta=beta.cuda(),
                                             initial_state=s0.cuda(), output_final_state=True)
    ref = oracle(q, k, v, g, beta, do, h0=s0, dht=dht)
    assert rel_l2(np64(o), ref["o"]) < 1e-5
    assert rel_l2(np64(ht), ref["final_state"]) < 1e-5
