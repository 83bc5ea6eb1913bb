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
