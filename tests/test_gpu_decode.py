"""GPU parity of the recurrent (decode) form: a prefix summarised as a state, then new tokens one
at a time and in chunks, must give the rows of the flash attention over the whole sequence
(bf16: relative L2 <= 1e-2, the tensor-core tolerance), and the state extended step by step must
equal the state of all tokens at once."""

from __future__ import annotations

import pytest
import torch

from oracle.kata_oracle import rel_l2

pytestmark = pytest.mark.gpu


def _draw(B, T, H, D, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=g) / D ** 0.5
    k = torch.randn(B, T, H, D, generator=g)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(B, T, H, D, generator=g)
    return (x.bfloat16().cuda() for x in (q, k, v))


@pytest.mark.parametrize("B,T0,H,D,M", [(2, 300, 2, 128, 4), (1, 129, 3, 64, 2)])
def test_decode_steps_match_full_attention(B, T0, H, D, M):
    from linatt_b200.kata_decode import kata_attn_state, kata_attn_step
    from linatt_b200.parallel_kata_attn import parallel_kata_attn

    chunks = [1, 7, 32, 1]
    T = T0 + sum(chunks)
    q, k, v = _draw(B, T, H, D, seed=T0 + D)
    with torch.no_grad():
        full = parallel_kata_attn(q, k, v, num_groups=M)
    state = kata_attn_state(k[:, :T0], v[:, :T0], num_groups=M)
    t = T0
    for n in chunks:
        o, state = kata_attn_step(q[:, t:t + n], k[:, t:t + n], v[:, t:t + n], state, num_groups=M)
        assert o.shape == (B, n, H, D) and o.dtype == v.dtype
        e = rel_l2(o.float().cpu().numpy(), full[:, t:t + n].float().cpu().numpy())
        assert e < 1e-2, f"tokens [{t}, {t + n}): rel-L2 {e:.3e}"
        t += n
    whole = kata_attn_state(k, v, num_groups=M)
    e = rel_l2(state.cpu().numpy(), whole.cpu().numpy())
    assert e < 1e-5, f"state rel-L2 {e:.3e}"


def test_decode_without_prefix_is_the_flash_forward():
    from linatt_b200.kata_decode import kata_attn_step
    from linatt_b200.parallel_kata_attn import parallel_kata_attn

    q, k, v = _draw(1, 50, 2, 128, seed=5)
    o, state = kata_attn_step(q, k, v, None, num_groups=4)
    with torch.no_grad():
        ref = parallel_kata_attn(q, k, v, num_groups=4)
    assert torch.equal(o, ref)
    assert state.shape == (2, 4 * 32 * 32, 136)


def _psi(x, M, scale):
    """psi(x) (N, F) fp32 of rows x (N, D): scale * x_{g,a} x_{g,b}, (g, a, b) row-major."""
    N, D = x.shape
    xg = x.float().view(N, M, D // M)
    return (scale * (xg[:, :, :, None] * xg[:, :, None, :])).reshape(N, -1)


def _decode_ref(q, k, v, S, M, scale):
    """Plain torch fp32 statement of one decode step: S + psi(k)[v|1], then psi(q)^T S / y'."""
    B, H, D = q.shape
    Dv = v.shape[-1]
    pq, pk = _psi(q.reshape(B * H, D), M, scale), _psi(k.reshape(B * H, D), M, scale)
    v1 = torch.zeros(B * H, S.shape[-1], device=S.device)
    v1[:, :Dv] = v.reshape(B * H, Dv).float()
    v1[:, Dv] = 1.0
    Sn = S + pk[:, :, None] * v1[:, None, :]
    xy = torch.einsum("nf,nfc->nc", pq, Sn)
    y = xy[:, Dv]
    o = xy[:, :Dv] / torch.where(y > 0, y, torch.ones_like(y))[:, None]
    return o.reshape(B, H, Dv), y.reshape(B, H), Sn


@pytest.mark.parametrize("B,T0,H,D,Dv,M", [(2, 200, 3, 128, 128, 4), (1, 64, 1, 128, 128, 4),
                                           (3, 77, 2, 64, 96, 2), (4, 33, 5, 64, 64, 4)])
def test_decode_kernel_vs_torch_fp32(B, T0, H, D, Dv, M):
    from linatt_b200.kata_decode import kata_attn_decode, kata_attn_state

    g = torch.Generator().manual_seed(B * 1000 + D + Dv)
    k0 = torch.randn(B, T0, H, D, generator=g).cuda()
    v0 = torch.randn(B, T0, H, Dv, generator=g).cuda()
    S = kata_attn_state(k0, v0, num_groups=M)
    q, k = (torch.randn(B, H, D, generator=g).cuda() for _ in range(2))
    v = torch.randn(B, H, Dv, generator=g).cuda()
    scale = 1.0 / (D // M) ** 0.5
    o_ref, y_ref, S_ref = _decode_ref(q, k, v, S, M, scale)
    o, y = kata_attn_decode(q, k, v, S, num_groups=M, return_den=True)
    assert rel_l2(S.cpu().numpy(), S_ref.cpu().numpy()) < 1e-6
    assert rel_l2(y.cpu().numpy(), y_ref.cpu().numpy()) < 1e-5
    assert rel_l2(o.cpu().numpy(), o_ref.cpu().numpy()) < 1e-5
    # the padding columns of the state stay zero
    assert torch.count_nonzero(S[..., Dv + 1:]) == 0


@pytest.mark.parametrize("B,T0,H,D,M,dtype", [(2, 300, 2, 128, 4, torch.bfloat16), (1, 129, 3, 64, 2, torch.float16)])
def test_decode_kernel_steps_match_full_attention(B, T0, H, D, M, dtype):
    from linatt_b200.kata_decode import kata_attn_decode, kata_attn_state
    from linatt_b200.parallel_kata_attn import parallel_kata_attn

    steps = 8
    q, k, v = (x.to(dtype) for x in _draw(B, T0 + steps, H, D, seed=7 * T0 + D))
    with torch.no_grad():
        full = parallel_kata_attn(q, k, v, num_groups=M)
    S = kata_attn_state(k[:, :T0], v[:, :T0], num_groups=M)
    for t in range(T0, T0 + steps):
        o = kata_attn_decode(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], S, num_groups=M)
        assert o.shape == (B, 1, H, D) and o.dtype == dtype
        e = rel_l2(o.float().cpu().numpy(), full[:, t:t + 1].float().cpu().numpy())
        assert e < 1e-2, f"token {t}: rel-L2 {e:.3e}"
    whole = kata_attn_state(k, v, num_groups=M)
    assert rel_l2(S.cpu().numpy(), whole.cpu().numpy()) < 1e-2


def test_decode_kernel_zero_query_gives_zero_output():
    from linatt_b200.kata_decode import kata_attn_decode, kata_attn_state

    q, k, v = _draw(2, 20, 2, 128, seed=11)
    S = kata_attn_state(k[:, :19], v[:, :19], num_groups=4)
    o, y = kata_attn_decode(torch.zeros_like(q[:, 19]), k[:, 19], v[:, 19], S, num_groups=4, return_den=True)
    assert torch.count_nonzero(o) == 0 and torch.count_nonzero(y) == 0


def test_decode_kernel_rejects_bad_state():
    from linatt_b200.kata_decode import kata_attn_decode

    q, k, v = _draw(1, 1, 2, 128, seed=3)
    bad = torch.zeros(2, 4096, 128, device="cuda")  # ldw < Dv + 1
    with pytest.raises(ValueError):
        kata_attn_decode(q, k, v, bad, num_groups=4)
