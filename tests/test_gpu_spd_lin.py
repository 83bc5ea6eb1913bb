"""GPU parity of the head-major O(T) siblings of the delta rule: ``spd_state_lin`` (linear SPD
numerator, trainable) and ``spd_chunk_scan`` (normalised sum-score forward), against the fp64
restatement (oracle/delta_oracle.py) and against the reference's own Triton kernels run on a B200
(tests/golden/spd_golden_gpu.npz, made by tests/golden/make_golden_delta_gpu.py --what spd).
Tolerances (relative L2): 1e-5 for fp32 inputs (fp32-exact kernels), 1e-2 for bf16 inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import delta_oracle as do_
from oracle.kata_oracle import rel_l2

pytestmark = pytest.mark.gpu


def draw(seed, B, H, T, D, Dv, dtype):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, H, T, D, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, H, T, D, generator=g), dim=-1)
    v = torch.randn(B, H, T, Dv, generator=g)
    do = torch.randn(B, H, T, Dv, generator=g)
    return tuple(x.to(dtype) for x in (q, k, v)) + (do,)


SHAPES = [(1, 2, 200, 64, 64, 4, 0.5), (2, 1, 64, 32, 32, 2, None), (1, 3, 130, 128, 128, 4, None)]


# T = 1 is checked in fp32 only: a single row's gradient is one dot product, whose relative error
# after rounding dO and the result to bf16 is not an rms figure over many rows
@pytest.mark.parametrize("dtype,tol,B,H,T,D,Dv,M,scale",
                         [(torch.float32, 1e-5) + s for s in SHAPES + [(1, 1, 1, 64, 32, 1, 0.5)]]
                         + [(torch.bfloat16, 1e-2) + s for s in SHAPES])
def test_spd_state_lin_matches_oracle(dtype, tol, B, H, T, D, Dv, M, scale):
    from linatt_b200.spd import spd_state_lin

    q, k, v, do = draw(B * T + M, B, H, T, D, Dv, dtype)
    leaves = [x.cuda().requires_grad_(True) for x in (q, k, v)]
    o = spd_state_lin(*leaves, M, scale=scale)
    assert o.dtype == torch.float32 and o.shape == (B, H, T, Dv)
    o.backward(do.cuda())
    f = lambda x: x.double().numpy()  # noqa: E731
    ref = do_.state_lin(f(q), f(k), f(v), M, scale=scale, grad_out=f(do))
    got = dict(o=o.detach(), dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad)
    for name, x in got.items():
        if name != "o":
            assert x.dtype == dtype
        e = rel_l2(x.float().cpu().double().numpy(), ref[name])
        assert e < tol, f"{name}: rel-L2 {e:.3e}"


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
def test_spd_chunk_scan_matches_oracle(dtype, tol):
    from linatt_b200.spd import spd_chunk_scan

    B, H, T, D, M = 2, 2, 192, 64, 4
    q, k, v, _ = draw(5, B, H, T, D, D, dtype)
    o, den = spd_chunk_scan(q.cuda(), k.cuda(), v.cuda(), M, "sum", scale=0.5)
    assert o.dtype == dtype and den.dtype == torch.float32 and den.shape == (B, H, T)
    ref = do_.chunk_scan(q.double().numpy(), k.double().numpy(), v.double().numpy(), M, scale=0.5)
    assert rel_l2(o.float().cpu().double().numpy(), ref["o"]) < tol
    assert rel_l2(den.cpu().double().numpy(), ref["den"]) < (1e-5 if dtype == torch.float32 else 1e-3)
    # eps clamp: a zero query row has den = eps and o = 0
    q0 = q.clone()
    q0[:, :, 0] = 0
    o0, den0 = spd_chunk_scan(q0.cuda(), k.cuda(), v.cuda(), M, "sum", scale=0.5, eps=1e-6)
    assert torch.all(den0[:, :, 0] == 1e-6) and torch.all(o0[:, :, 0] == 0)
    with pytest.raises(ValueError):
        spd_chunk_scan(q.cuda(), k.cuda(), v.cuda(), M, "concat")


def _spd_golden():
    from tests.conftest import GOLDEN

    path = GOLDEN / "spd_golden_gpu.npz"
    z = np.load(path)
    out = {}
    for key in z.files:
        if "/" in key:
            case, name = key.split("/")
            out.setdefault(case, {})[name] = z[key]
    return out


@pytest.mark.parametrize("case", ["scan_m4", "scan_m2_default_scale"])
def test_head_major_siblings_match_reference_run_on_gpu(case):
    """spd_chunk_scan against the reference's Triton kernels on a B200, same bf16 inputs (rel-L2 <=
    1e-2, the bf16 bar; the reference rounds its dot operands to bf16)."""
    from linatt_b200.spd import flash_delta_state, spd_chunk_scan, spd_state_lin

    rec = _spd_golden()[case]
    B, H, T, D, Dv, M, scale = rec["meta"]
    M, scale, fn = int(M), (None if scale < 0 else float(scale)), str(rec["fn"])
    t = lambda x, dt=torch.bfloat16: torch.from_numpy(x).to(dt).cuda()  # noqa: E731
    q, k, v, beta = t(rec["q"]), t(rec["k"]), t(rec["v"]), t(rec["beta"])
    if fn == "chunk_scan":
        o, den = spd_chunk_scan(q, k, v, M, "sum", scale=scale)
        got = dict(o=o, den=den)
    else:
        leaves = [x.clone().requires_grad_(True) for x in ((q, k, v) if fn == "state_lin" else (q, k, v, beta))]
        f = spd_state_lin if fn == "state_lin" else flash_delta_state
        o = f(*leaves, M, scale=scale)
        o.backward(t(rec["do"], o.dtype))
        got = dict(o=o.detach(), dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad)
        if fn == "delta_state":
            got["dbeta"] = leaves[3].grad
    for name, x in got.items():
        e = rel_l2(x.float().cpu().double().numpy(), rec[name])
        assert e < 1e-2, f"{case} {name}: rel-L2 {e:.3e}"


@pytest.mark.parametrize("case", ["m4_raw", "m1_raw"])
def test_flash_delta_state_matches_reference_flash_delta_run_on_gpu(golden_delta_gpu, case):
    """flash_delta_state is the raw-numerator delta rule in head-major layout.  The reference's own
    kernel for it (kata/spd/chunk_state_v2.py) asks for more tensor memory than a B200 has, so it is
    pinned against the reference's flash_delta (normalize=False) run on a B200 on the same inputs,
    transposed to head-major: o and dq, dk, dv, dbeta (rel-L2 <= 1e-2)."""
    from linatt_b200.spd import flash_delta_state

    rec = golden_delta_gpu[case]
    B, T, H, D, Dv, M, scale, norm = rec["meta"]
    assert not norm
    M, scale = int(M), (None if scale < 0 else float(scale))
    hm = lambda x, dt=torch.bfloat16: torch.from_numpy(x).to(dt).cuda().transpose(1, 2).contiguous()  # noqa: E731
    leaves = [hm(rec[n]).requires_grad_(True) for n in ("q", "k", "v", "beta")]
    o = flash_delta_state(*leaves, M, scale=scale)
    o.backward(hm(rec["do"], torch.float32))
    got = dict(o=o.detach(), dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad, dbeta=leaves[3].grad)
    for name, x in got.items():
        e = rel_l2(x.transpose(1, 2).float().cpu().double().numpy(), rec[name])
        assert e < 1e-2, f"{case} {name}: rel-L2 {e:.3e}"


@pytest.mark.parametrize("case", ["m4_norm", "m4_raw", "m2_norm_default_scale", "m1_raw"])
def test_spd_state_lin_matches_reference_readout_run_on_gpu(golden_delta_gpu, case):
    """spd_state_lin's numerator is tril(kappa(q, k)) v.  The reference's own kernel for it
    (kata/spd/chunk_state_lin.py) asks for more tensor memory than a B200 has, so it is pinned
    against the reference's flash_delta_readout run on a B200, which computes the same numerator of
    its U: our spd_state_lin(q, k, U) (head-major) against the fixture's num (rel-L2 <= 1e-2)."""
    from linatt_b200.spd import spd_state_lin

    rec = golden_delta_gpu[case]
    B, T, H, D, Dv, M, scale, norm = rec["meta"]
    M, scale = int(M), (None if scale < 0 else float(scale))
    hm = lambda x, dt: torch.from_numpy(x).to(dt).cuda().transpose(1, 2).contiguous()  # noqa: E731
    o = spd_state_lin(hm(rec["q"], torch.bfloat16), hm(rec["k"], torch.bfloat16), hm(rec["U"], torch.float32), M,
                      scale=scale)
    e = rel_l2(o.transpose(1, 2).float().cpu().double().numpy(), rec["num"])
    assert e < 1e-2, f"{case}: rel-L2 {e:.3e}"
