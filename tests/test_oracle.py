"""The CPU oracle against the golden fixtures produced by the reference's own code."""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import kata_oracle as ko
from tests.conftest import attn_case_meta

ATTN_CASES = ["concat_m1", "concat_m2", "concat_m4", "concat_m4_d128", "sum_m2", "sum_m4", "decay_m2",
              "decay_m4", "gqa_m2"]


@pytest.mark.parametrize("case", ATTN_CASES)
def test_oracle_forward_matches_reference(golden, case):
    rec = golden[case]
    m = attn_case_meta(rec)
    scale = 1.0 / math.sqrt(m["D"] // m["M"])
    o, den = ko.attn_fwd(rec["q"], rec["k"], rec["v"], m["M"], scale, m["score"], rec.get("c"))
    # Triton K1/K2 (interpreter, fp32) and the float64 torch reference
    assert ko.rel_l2(o, rec["o"]) < 2e-6
    assert ko.rel_l2(den, rec["den"]) < 2e-6
    if "o_ref64" in rec:
        assert ko.rel_l2(o, rec["o_ref64"]) < 1e-6


@pytest.mark.parametrize("case", ATTN_CASES)
def test_oracle_backward_matches_reference(golden, case):
    rec = golden[case]
    m = attn_case_meta(rec)
    scale = 1.0 / math.sqrt(m["D"] // m["M"])
    dq, dk, dv, dc = ko.attn_bwd(rec["q"], rec["k"], rec["v"], rec["do"], m["M"], scale, m["score"], rec.get("c"))
    for name, x in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert ko.rel_l2(x, rec[name]) < 2e-6, name
    if m["decay"]:
        assert ko.rel_l2(dc, rec["dc"]) < 2e-6


def test_oracle_offset_gate_matches_reference(golden):
    rec = golden["offset_m2"]
    M, E = (int(x) for x in rec["meta"])
    qi, ki = ko.augment_offset(rec["q"], rec["k"], rec["off"], M)
    np.testing.assert_array_equal(qi.astype(np.float32), rec["q_in"])
    np.testing.assert_array_equal(ki.astype(np.float32), rec["k_in"])


def test_oracle_backward_is_gradient_of_forward():
    """Finite-difference check of the closed-form backward (independent of the fixtures)."""
    rng = np.random.default_rng(3)
    B, T, H, D, M = 1, 9, 1, 8, 2
    q, k, v, do = (rng.standard_normal((B, T, H, D)) for _ in range(4))
    c = np.cumsum(-np.log1p(np.exp(rng.standard_normal((B, T, H)))), axis=1)
    for score, cc in (("concat", None), ("sum", None), ("concat", c)):
        dq, dk, dv, dc = ko.attn_bwd(q, k, v, do, M, 0.7, score, cc)

        def f(qq, kk, vv, c2):
            return float((ko.attn_fwd(qq, kk, vv, M, 0.7, score, c2)[0] * do).sum())

        eps = 1e-6
        for arr, grad, idx in ((q, dq, (0, 5, 0, 3)), (k, dk, (0, 2, 0, 6)), (v, dv, (0, 1, 0, 0))):
            xp = arr.copy()
            xp[idx] += eps
            xm = arr.copy()
            xm[idx] -= eps
            args_p = [xp if a is arr else a for a in (q, k, v)]
            args_m = [xm if a is arr else a for a in (q, k, v)]
            num = (f(*args_p, cc) - f(*args_m, cc)) / (2 * eps)
            assert abs(num - grad[idx]) < 1e-6 * max(1.0, abs(num))
        if cc is not None:
            cp = cc.copy()
            cp[0, 4, 0] += eps
            cm = cc.copy()
            cm[0, 4, 0] -= eps
            num = (f(q, k, v, cp) - f(q, k, v, cm)) / (2 * eps)
            assert abs(num - dc[0, 4, 0]) < 1e-6 * max(1.0, abs(num))


# ------------------------------------------------------------------------------------------------
# SPD delta rule
# ------------------------------------------------------------------------------------------------
def _delta_golden():
    from tests.conftest import GOLDEN

    z = np.load(GOLDEN / "delta_golden.npz")
    out = {}
    for key in z.files:
        case, name = key.split("/")
        out.setdefault(case, {})[name] = z[key]
    return out


@pytest.mark.parametrize("case", ["m1", "m2", "m4_default_scale"])
def test_delta_oracle_matches_reference_U(case):
    from oracle import delta_oracle as do

    rec = _delta_golden()[case]
    B, T, H, D, Dv, M, scale = rec["meta"]
    scale = None if scale < 0 else float(scale)
    res = do.flash_delta(rec["q"], rec["k"], rec["v"], rec["beta"], int(M), scale)
    assert ko.rel_l2(res["U"], rec["U"]) < 1e-5
    # erase term identity: beta * (V - E) = U
    assert ko.rel_l2(rec["beta"][..., None] * (rec["v"] - res["E"]), res["U"]) < 1e-10


@pytest.mark.parametrize("case", ["m4_norm", "m4_raw", "m2_norm_default_scale", "m1_raw"])
def test_delta_oracle_matches_reference_run_on_gpu(case):
    """The whole delta rule against the reference's own Triton flash_delta run on a B200
    (tests/golden/make_golden_delta_gpu.py): multi-chunk U, the readout numerator, den, o for both
    normalize settings, and dq, dk, dv, dbeta.  The reference casts its inter-chunk products and
    readout operands to bf16 and returns bf16 gradients, so it sits a few 1e-3 (rel-L2) from the
    exact fp64 restatement: the tolerance is the bf16 bar, 1e-2."""
    from oracle import delta_oracle as do
    from tests.conftest import load_delta_gpu_golden

    rec = load_delta_gpu_golden()[case]
    B, T, H, D, Dv, M, scale, norm = rec["meta"]
    scale = None if scale < 0 else float(scale)
    raw = do.flash_delta(rec["q"], rec["k"], rec["v"], rec["beta"], int(M), scale)
    full = do.flash_delta(rec["q"], rec["k"], rec["v"], rec["beta"], int(M), scale, normalize=bool(norm),
                          eps=1e-5, grad_out=rec["do"])
    pairs = [("U", raw["U"]), ("num", raw["o"]), ("den", raw["den"]), ("o", full["o"])]
    pairs += [(g, full[g]) for g in ("dq", "dk", "dv", "dbeta")]
    for name, ref in pairs:
        e = ko.rel_l2(ref, rec[name])
        assert e < 1e-2, f"{case} {name}: rel-L2 {e:.3e}"


def test_delta_oracle_gradients_finite_difference():
    from oracle import delta_oracle as do

    rng = np.random.default_rng(5)
    B, T, H, D, M = 1, 11, 1, 8, 2
    q, k, v = (rng.standard_normal((B, T, H, D)) for _ in range(3))
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, H))))
    go = rng.standard_normal((B, T, H, D))
    for normalize in (False, True):
        res = do.flash_delta(q, k, v, beta, M, 0.5, normalize, grad_out=go)

        def f(qq, kk, vv, bb):
            return float((do.flash_delta(qq, kk, vv, bb, M, 0.5, normalize)["o"] * go).sum())

        eps = 1e-6
        for arr, gname, idx in ((q, "dq", (0, 6, 0, 3)), (k, "dk", (0, 2, 0, 5)), (v, "dv", (0, 4, 0, 1)),
                                (beta, "dbeta", (0, 3, 0))):
            xp, xm = arr.copy(), arr.copy()
            xp[idx] += eps
            xm[idx] -= eps
            args_p = [xp if a is arr else a for a in (q, k, v, beta)]
            args_m = [xm if a is arr else a for a in (q, k, v, beta)]
            num = (f(*args_p) - f(*args_m)) / (2 * eps)
            assert abs(num - res[gname][idx]) < 1e-6 * max(1.0, abs(num)), gname


# ------------------------------------------------------------------------------------------------
# Gated delta rule (fla chunk_gated_delta_rule)
# ------------------------------------------------------------------------------------------------
def _gdn_golden():
    from tests.conftest import GOLDEN

    z = np.load(GOLDEN / "gdn_golden.npz")
    out = {}
    for key in z.files:
        case, name = key.split("/")
        out.setdefault(case, {})[name] = z[key]
    return out


@pytest.mark.parametrize("case", ["basic", "chunk_t128", "varlen"])
def test_gdn_oracle_matches_fla_naive(case):
    from oracle import gdn_oracle as go

    rec = _gdn_golden()[case]
    res = go.gdn(rec["q"], rec["k"], rec["v"], rec["g"], rec["beta"], initial_state=rec.get("h0"),
                 output_final_state=True, cu_seqlens=rec.get("cu_seqlens"), grad_out=rec["do"],
                 grad_final=rec["dht"])
    assert ko.rel_l2(res["o"], rec["o"]) < 1e-5
    assert ko.rel_l2(res["final_state"], rec["ht"]) < 1e-5
    for n in ("dq", "dk", "dv", "dg", "dbeta") + (("dh0",) if "h0" in rec else ()):
        assert ko.rel_l2(res[n], rec[n]) < 1e-5, n
    if "o_chunk" in rec:  # fla's chunked naive form agrees with its recurrent form
        assert ko.rel_l2(rec["o_chunk"], rec["o"]) < 1e-5


def test_gdn_oracle_gate_and_l2norm_finite_difference():
    """The in-kernel gate and q/k l2norm options: gradients of the oracle against central
    differences (the options are prologue transforms; fla's formulas are restated)."""
    from oracle import gdn_oracle as go

    rng = np.random.default_rng(7)
    B, T, H, HV, K, V = 1, 9, 1, 2, 4, 3
    q, k = (rng.standard_normal((B, T, H, K)) for _ in range(2))
    v = rng.standard_normal((B, T, HV, V))
    g = rng.standard_normal((B, T, HV))
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))
    A_log, dt_bias = rng.standard_normal(HV) * 0.3, rng.standard_normal(HV) * 0.3
    do_ = rng.standard_normal((B, T, HV, V))
    kw = dict(use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=A_log, dt_bias=dt_bias)
    res = go.gdn(q, k, v, g, beta, grad_out=do_, **kw)

    def f(**over):
        args = dict(q=q, k=k, v=v, g=g, beta=beta, **kw)
        args.update(over)
        return float((go.gdn(**args)["o"] * do_).sum())

    eps = 1e-6
    for name, arr, idx in (("q", q, (0, 5, 0, 2)), ("k", k, (0, 3, 0, 1)), ("g", g, (0, 4, 1)),
                           ("A_log", A_log, (1,)), ("dt_bias", dt_bias, (0,))):
        xp, xm = arr.copy(), arr.copy()
        xp[idx] += eps
        xm[idx] -= eps
        num = (f(**{name: xp}) - f(**{name: xm})) / (2 * eps)
        assert abs(num - res["d" + name][idx]) < 1e-6 * max(1.0, abs(num)), name


def test_tail_window_oracle_matches_the_full_oracle():
    """attn_tail_window (used for the config-4 check at T = 131072) is exact for the last w rows."""
    rng = np.random.default_rng(1)
    T, D, w = 300, 64, 40
    q, k, v, do = (rng.standard_normal((1, T, 1, D)) / 8 for _ in range(4))
    o, den = ko.attn_fwd(q, k, v, 4)
    dq, dk, dv, _ = ko.attn_bwd(q, k, v, do, 4)
    r = ko.attn_tail_window(q[0, :, 0], k[0, :, 0], v[0, :, 0], do[0, :, 0], 4, w, chunk=64)
    for name, full in (("o", o), ("den", den), ("dq", dq), ("dk", dk), ("dv", dv)):
        assert ko.rel_l2(r[name], full[0, -w:, 0]) < 1e-12, name
