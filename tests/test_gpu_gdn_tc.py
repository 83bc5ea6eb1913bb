"""GPU parity of the tensor-core (tcgen05) gated delta rule, the kernels that bf16 / fp16 inputs take.

Each case runs the same 16-bit inputs through the tcgen05 kernels and checks outputs and every
gradient against the fp64 oracle on those 16-bit values (rel-L2 <= 1e-2, the bf16 bar), and
against the fp32-exact CUDA-core kernels forced on the same inputs.  Covers grouped value heads,
initial / final states, ragged T (a partial last chunk), narrow heads (zero-padded), varlen
sequences, fp16, the gate / l2norm options, and the backward without the forward's workspace."""

from __future__ import annotations

import pytest
import torch

from oracle.kata_oracle import rel_l2
from tests.test_gpu_gdn import GRADS, draw, np64, oracle, run

pytestmark = pytest.mark.gpu


@pytest.fixture
def algo(monkeypatch):
    from linatt_b200 import gated_delta_rule as gdr

    def set_algo(name):
        monkeypatch.setattr(gdr, "ALGO", name)

    return set_algo


CASES = [
    # B, T, H, HV, K, V, h0, dtype
    (2, 200, 2, 4, 64, 64, True, torch.bfloat16),
    (1, 64, 1, 1, 64, 64, False, torch.bfloat16),
    (1, 1, 1, 1, 64, 64, True, torch.bfloat16),
    (3, 130, 2, 2, 48, 40, True, torch.bfloat16),
    (2, 257, 3, 3, 64, 64, True, torch.float16),
]


@pytest.mark.parametrize("B,T,H,HV,K,V,h0,dtype", CASES)
def test_tc_matches_oracle_and_simt(algo, B, T, H, HV, K, V, h0, dtype):
    q, k, v, g, beta, do, s0, dht = draw(T + 3 * HV, B, T, H, HV, K, V, dtype=dtype, h0=h0)
    algo("tc")
    got = run(q, k, v, g, beta, do, h0=s0, dht=dht)
    assert got["o"].dtype == dtype
    ref = oracle(q, k, v, g, beta, do, h0=s0, dht=dht)
    algo("simt")
    exact = run(q, k, v, g, beta, do, h0=s0, dht=dht)
    names = [("o", "o"), ("ht", "final_state")] + [(n, n) for n in GRADS + (("dh0",) if h0 else ())]
    for n, r in names:
        e = rel_l2(np64(got[n]), ref[r])
        assert e < 1e-2, f"{n}: rel-L2 {e:.3e} against the oracle"
        e = rel_l2(np64(got[n]), np64(exact[n]))
        assert e < 1e-2, f"{n}: rel-L2 {e:.3e} against the fp32-exact kernels"


def test_tc_varlen_and_options(algo):
    algo("tc")
    cu = torch.tensor([0, 1, 65, 200, 333], dtype=torch.int64)
    T = int(cu[-1])
    q, k, v, g, beta, do, _, _ = draw(8, 1, T, 2, 2, 64, 64, dtype=torch.bfloat16)
    gen = torch.Generator().manual_seed(9)
    s0 = torch.randn(4, 2, 64, 64, generator=gen) * 0.1
    dht = torch.randn(4, 2, 64, 64, generator=gen) * 0.1
    got = run(q, k, v, g, beta, do, h0=s0, dht=dht, cu=cu)
    ref = oracle(q, k, v, g, beta, do, h0=s0, dht=dht, cu=cu)
    for n, r in [("o", "o"), ("ht", "final_state")] + [(n, n) for n in GRADS + ("dh0",)]:
        e = rel_l2(np64(got[n]), ref[r])
        assert e < 1e-2, f"varlen {n}: rel-L2 {e:.3e}"
    # gate in kernel + qk l2norm
    q, k, v, g, beta, do, s0, dht = draw(4, 1, 150, 2, 2, 64, 64, dtype=torch.bfloat16, h0=True)
    A_log = torch.randn(2) * 0.3
    dt_bias = torch.randn(2) * 0.3
    kw = dict(use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=A_log, dt_bias=dt_bias)
    got = run(q, k, v, g, beta, do, h0=s0, dht=dht, **dict(kw))
    ref = oracle(q, k, v, g, beta, do, h0=s0, dht=dht, **kw)
    for n, r in [("o", "o"), ("ht", "final_state")] + [(n, n) for n in GRADS + ("dh0",)]:
        e = rel_l2(np64(got[n]), ref[r])
        assert e < 1e-2, f"options {n}: rel-L2 {e:.3e}"
    # dA_log and ddt_bias have one entry per head: each is a sum over all 150 tokens of signed
    # per-token terms dg_t * dg_t/dtheta, so the bf16-level error of the per-token dg (held to 1e-2
    # above) does not shrink with the cancellation in that sum; they are held to 3e-2.
    for n in ("dA_log", "ddt_bias"):
        e = rel_l2(np64(got[n]), ref[n])
        assert e < 3e-2, f"options {n}: rel-L2 {e:.3e}"


def test_tc_backward_recompute_path_matches_reuse(algo):
    """Without the forward's workspace the tensor-core backward rebuilds W, U0, u and the chunk states
    from the saved A; the 16-bit operands are rounded from the same fp32 values, so the gradients
    agree with the reuse path to fp32 rounding."""
    from linatt_b200 import gated_delta_rule as gdr

    algo("tc")
    B, T, H, K, V = 2, 300, 2, 64, 64
    q, k, v, g, beta, do, s0, dht = draw(12, B, T, H, H, K, V, dtype=torch.bfloat16, h0=True)
    qc, kc, vc, gc, bc, s0c, dhtc = (x.cuda().contiguous() for x in (q, k, v, g, beta, s0, dht))
    doc = do.to(torch.bfloat16).cuda().contiguous()
    tables = gdr._chunk_tables(None, None, B, T, qc.device)
    o, A, ht, ws = gdr._fwd(qc, kc, vc, gc, bc, K ** -0.5, s0c, True, tables)
    a = gdr._bwd(qc, kc, vc, gc, bc, A, K ** -0.5, s0c, doc, dhtc, tables, fwd_ws=ws)
    b = gdr._bwd(qc, kc, vc, gc, bc, A, K ** -0.5, s0c, doc, dhtc, tables, fwd_ws=None)
    for x, y in zip(a, b):
        assert rel_l2(np64(x), np64(y)) < 1e-6


def test_tc_refuses_fp32_inputs(algo):
    algo("tc")
    q, k, v, g, beta, do, _, _ = draw(1, 1, 64, 1, 1, 64, 64)
    with pytest.raises(RuntimeError):
        run(q, k, v, g, beta, do)
