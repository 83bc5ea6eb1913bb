"""GPU parity of the recurrent (decode) form.  A prefix summarised as a state, then new tokens one
at a time (the fused ``kata_decode_step`` kernel) and in chunks, must give the rows of the flash
attention over the whole sequence (bf16: relative L2 <= 1e-2, the tensor-core tolerance), for the
concat and sum scores, GQA and the decayed form.  The state extended step by step must equal the
state of all tokens at once.  One kernel step must also match a plain torch fp32 statement of the
step (state 1e-6, outputs 1e-5)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle.kata_oracle import rel_l2

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return rel_l2(a.float().cpu().numpy(), b.float().cpu().numpy())


def _draw(B, T, HQ, H, D, seed, dtype=torch.bfloat16, decay=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, HQ, D, generator=g) / D ** 0.5
    k = F.normalize(torch.randn(B, T, H, D, generator=g), dim=-1)
    v = torch.randn(B, T, H, D, generator=g)
    lg = -0.2 * F.softplus(torch.randn(B, T, HQ, generator=g)) if decay else None
    out = [x.to(dtype).cuda() for x in (q, k, v)]
    return out + [None if lg is None else lg.cuda()]


def _full(q, k, v, M, score, lg):
    from linatt_b200.parallel_kata_attn import parallel_kata_attn, parallel_kata_attn_decay, parallel_kata_attn_sum

    with torch.no_grad():
        if lg is not None:
            return parallel_kata_attn_decay(q, k, v, torch.cumsum(lg, 1), num_groups=M)
        if score == "sum":
            return parallel_kata_attn_sum(q, k, v, num_groups=M)
        return parallel_kata_attn(q, k, v, num_groups=M)


CASES = [  # B, T0, HQ, H, D, M, score, decay
    (2, 300, 2, 2, 128, 4, "concat", False),
    (1, 129, 3, 3, 64, 2, "concat", False),
    (2, 200, 4, 2, 128, 4, "concat", False),
    (2, 150, 2, 2, 128, 4, "sum", False),
    (1, 100, 4, 1, 64, 2, "sum", False),
    (2, 180, 4, 2, 128, 2, "concat", True),
]


@pytest.mark.parametrize("B,T0,HQ,H,D,M,score,decay", CASES)
def test_decode_chunks_match_full_attention(B, T0, HQ, H, D, M, score, decay):
    from linatt_b200.kata_decode import kata_attn_state, kata_attn_step

    chunks = [1, 7, 32, 1]
    T = T0 + sum(chunks)
    q, k, v, lg = _draw(B, T, HQ, H, D, seed=T0 + D, decay=decay)
    full = _full(q, k, v, M, score, lg)
    c0 = None if lg is None else torch.cumsum(lg[:, :T0], 1)
    state = kata_attn_state(k[:, :T0], v[:, :T0], num_groups=M, score=score, c=c0, HQ=HQ)
    t = T0
    for n in chunks:
        gi = None if lg is None else lg[:, t:t + n]
        o, state = kata_attn_step(q[:, t:t + n], k[:, t:t + n], v[:, t:t + n], state, num_groups=M, score=score,
                                  g=gi)
        assert o.shape == (B, n, HQ, D) and o.dtype == v.dtype
        e = _rel(o, full[:, t:t + n])
        assert e < 1e-2, f"tokens [{t}, {t + n}): rel-L2 {e:.3e}"
        t += n
    whole = kata_attn_state(k, v, num_groups=M, score=score, c=None if lg is None else torch.cumsum(lg, 1), HQ=HQ)
    e = _rel(state, whole)
    assert e < 1e-2, f"state rel-L2 {e:.3e}"


def test_decode_without_prefix_is_the_flash_forward():
    from linatt_b200.kata_decode import kata_attn_step

    q, k, v, _ = _draw(1, 50, 2, 2, 128, seed=5)
    o, state = kata_attn_step(q, k, v, None, num_groups=4)
    assert torch.equal(o, _full(q, k, v, 4, "concat", None))
    assert state.shape == (2, 4 * 32 * 32, 136)


def _psi(x, M, scale, score):
    """psi(x) (N, F) fp32 of rows x (N, D)."""
    N, D = x.shape
    xg = x.float().view(N, M, D // M)
    if score == "sum":
        return (scale * torch.einsum("nga,ngb->nab", xg, xg)).reshape(N, -1)
    return (scale * (xg[:, :, :, None] * xg[:, :, None, :])).reshape(N, -1)


def _decode_ref(q, k, v, S, M, scale, score, lg):
    """Plain torch fp32 statement of one decode step: S <- exp(g) S + psi(k)[v|1], then psi(q)^T S / y'."""
    B, HQ, D = q.shape
    H, Dv = k.shape[1], v.shape[-1]
    G, lds = HQ // H, S.shape[-1]
    pk = _psi(k.reshape(B * H, D), M, scale, score)
    Fn = pk.shape[1]
    v1 = torch.zeros(B * H, lds, device=S.device)
    v1[:, :Dv] = v.reshape(B * H, Dv).float()
    v1[:, Dv] = 1.0
    upd = pk[:, :, None] * v1[:, None, :]
    pq = _psi(q.reshape(B * HQ, D), M, scale, score)
    if lg is None:
        Sn = S + upd
        xy = torch.einsum("bhjf,bhfc->bhjc", pq.view(B, H, G, Fn), Sn.view(B, H, Fn, lds)).reshape(B * HQ, lds)
    else:
        updq = upd.view(B, H, 1, Fn, lds).expand(B, H, G, Fn, lds).reshape(B * HQ, Fn, lds)
        Sn = torch.exp(lg).reshape(B * HQ, 1, 1) * S + updq
        xy = torch.einsum("nf,nfc->nc", pq, Sn)
    y = xy[:, Dv]
    o = xy[:, :Dv] / torch.where(y > 0, y, torch.ones_like(y))[:, None]
    return o.reshape(B, HQ, Dv), y.reshape(B, HQ), Sn


@pytest.mark.parametrize("B,T0,HQ,H,D,Dv,M,score,decay", [
    (2, 200, 3, 3, 128, 128, 4, "concat", False),
    (1, 64, 1, 1, 128, 128, 4, "concat", False),
    (3, 77, 2, 2, 64, 96, 2, "concat", False),
    (4, 33, 5, 5, 64, 64, 4, "concat", False),
    (2, 50, 4, 2, 128, 128, 4, "concat", False),
    (1, 40, 8, 1, 64, 64, 2, "concat", False),
    (2, 60, 2, 2, 128, 128, 4, "sum", False),
    (2, 60, 4, 1, 64, 64, 2, "sum", False),
    (2, 70, 4, 2, 128, 128, 2, "concat", True),
])
def test_decode_kernel_vs_torch_fp32(B, T0, HQ, H, D, Dv, M, score, decay):
    from linatt_b200.kata_decode import kata_attn_decode, kata_attn_state

    g = torch.Generator().manual_seed(B * 1000 + D + Dv + HQ)
    k0 = torch.randn(B, T0, H, D, generator=g).cuda()
    v0 = torch.randn(B, T0, H, Dv, generator=g).cuda()
    c0 = torch.cumsum(-F.softplus(torch.randn(B, T0, HQ, generator=g)), 1).cuda() if decay else None
    S = kata_attn_state(k0, v0, num_groups=M, score=score, c=c0, HQ=HQ)
    q = torch.randn(B, HQ, D, generator=g).cuda()
    k = torch.randn(B, H, D, generator=g).cuda()
    v = torch.randn(B, H, Dv, generator=g).cuda()
    lg = -F.softplus(torch.randn(B, HQ, generator=g)).cuda() if decay else None
    scale = 1.0 / (D // M) ** 0.5
    o_ref, y_ref, S_ref = _decode_ref(q, k, v, S, M, scale, score, lg)
    o, y = kata_attn_decode(q, k, v, S, num_groups=M, score=score, g=lg, return_den=True)
    assert _rel(S, S_ref) < 1e-6
    assert _rel(y, y_ref) < 1e-5
    assert _rel(o, o_ref) < 1e-5
    assert torch.count_nonzero(S[..., Dv + 1:]) == 0  # the padding columns of the state stay zero


@pytest.mark.parametrize("B,T0,HQ,H,D,M,score,decay,dtype", [
    (2, 300, 2, 2, 128, 4, "concat", False, torch.bfloat16),
    (1, 129, 3, 3, 64, 2, "concat", False, torch.float16),
    (2, 100, 8, 2, 64, 4, "concat", False, torch.bfloat16),
    (2, 150, 4, 2, 128, 4, "sum", False, torch.bfloat16),
    (2, 120, 4, 2, 128, 2, "concat", True, torch.bfloat16),
])
def test_decode_kernel_steps_match_full_attention(B, T0, HQ, H, D, M, score, decay, dtype):
    from linatt_b200.kata_decode import kata_attn_decode, kata_attn_state

    steps = 8
    q, k, v, lg = _draw(B, T0 + steps, HQ, H, D, seed=7 * T0 + D, dtype=dtype, decay=decay)
    full = _full(q, k, v, M, score, lg)
    c = None if lg is None else torch.cumsum(lg, 1)
    S = kata_attn_state(k[:, :T0], v[:, :T0], num_groups=M, score=score, c=None if c is None else c[:, :T0], HQ=HQ)
    for t in range(T0, T0 + steps):
        gi = None if lg is None else lg[:, t]
        o = kata_attn_decode(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], S, num_groups=M, score=score, g=gi)
        assert o.shape == (B, 1, HQ, D) and o.dtype == dtype
        e = _rel(o, full[:, t:t + 1])
        assert e < 1e-2, f"token {t}: rel-L2 {e:.3e}"
    whole = kata_attn_state(k, v, num_groups=M, score=score, c=c, HQ=HQ)
    assert _rel(S, whole) < 1e-2


def test_decode_kernel_zero_query_gives_zero_output():
    from linatt_b200.kata_decode import kata_attn_decode, kata_attn_state

    q, k, v, _ = _draw(2, 20, 2, 2, 128, seed=11)
    S = kata_attn_state(k[:, :19], v[:, :19], num_groups=4)
    o, y = kata_attn_decode(torch.zeros_like(q[:, 19]), k[:, 19], v[:, 19], S, num_groups=4, return_den=True)
    assert torch.count_nonzero(o) == 0 and torch.count_nonzero(y) == 0


def test_decode_kernel_rejects_bad_state():
    from linatt_b200.kata_decode import kata_attn_decode

    q, k, v, _ = _draw(1, 1, 2, 2, 128, seed=3)
    bad = torch.zeros(2, 4096, 128, device="cuda")  # ldw < Dv + 1
    with pytest.raises(ValueError):
        kata_attn_decode(q[:, 0], k[:, 0], v[:, 0], bad, num_groups=4)
    with pytest.raises(ValueError):  # decay with the sum score
        kata_attn_decode(q[:, 0], k[:, 0], v[:, 0], bad, num_groups=4, score="sum", g=torch.zeros(1, 2, device="cuda"))


@pytest.mark.parametrize("B,T,H,D,M,dtype", [(2, 37, 3, 128, 4, torch.bfloat16), (1, 70, 2, 64, 4, torch.float32),
                                             (2, 16, 1, 64, 1, torch.float16), (1, 5, 2, 128, 2, torch.bfloat16)])
def test_feature_kernel_is_exact(B, T, H, D, M, dtype):
    """psi(x) from the feature kernel equals the torch fp32 statement rounded to bf16, bit for bit."""
    from linatt_b200.kata_decode import state_features

    g = torch.Generator().manual_seed(T * D + M)
    x = torch.randn(B, T, H, D, generator=g).to(dtype).cuda()
    scale = 1.0 / (D // M) ** 0.5
    R = state_features(x, M, scale, "concat")
    ref = _psi(x.permute(0, 2, 1, 3).reshape(B * H * T, D), M, scale, "concat").to(torch.bfloat16)
    assert torch.equal(R.reshape(B * H * T, -1), ref)


@pytest.mark.parametrize("B,T,H,D,M,dtype", [(2, 37, 3, 128, 4, torch.bfloat16), (1, 70, 2, 64, 2, torch.float32),
                                             (2, 20, 1, 64, 4, torch.float16), (1, 5, 2, 256, 8, torch.bfloat16)])
def test_sum_feature_kernel_vs_torch(B, T, H, D, M, dtype):
    """The sum score's features scale * sum_g x_{g,a} x_{g,b} from the kernel against the torch fp32
    statement rounded to bf16 (only the fp32 summation order may differ: rel-L2 <= 1e-3)."""
    from linatt_b200.kata_decode import state_features

    g = torch.Generator().manual_seed(T * D + M + 1)
    x = torch.randn(B, T, H, D, generator=g).to(dtype).cuda()
    scale = 1.0 / (D // M) ** 0.5
    R = state_features(x, M, scale, "sum")
    ref = _psi(x.permute(0, 2, 1, 3).reshape(B * H * T, D), M, scale, "sum")
    assert R.shape == (B * H, T, (D // M) ** 2) and R.dtype == torch.bfloat16
    assert _rel(R.reshape(B * H * T, -1), ref.bfloat16()) < 1e-3
