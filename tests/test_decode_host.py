"""Host-side checks of the decode and varlen APIs (no GPU): CPU tensors are refused (there is no
CPU path), and bad arguments raise before anything reaches a device."""

import pytest
import torch

from linatt_b200.kata_decode import kata_attn_decode, kata_attn_state, kata_attn_step
from linatt_b200.varlen import parallel_kata_attn_varlen


def test_decode_refuses_cpu_tensors():
    q, k, v = torch.randn(1, 2, 64), torch.randn(1, 2, 64), torch.randn(1, 2, 64)
    state = torch.zeros(2, 4 * 16 * 16, 72)
    with pytest.raises(RuntimeError, match="CUDA"):
        kata_attn_decode(q, k, v, state, num_groups=4)


def test_decay_with_sum_score_is_rejected():
    x = torch.randn(1, 4, 2, 64)
    with pytest.raises(ValueError, match="concat"):
        kata_attn_state(x, x, num_groups=4, score="sum", c=torch.zeros(1, 4, 2))
    with pytest.raises(ValueError, match="concat"):
        kata_attn_step(x, x, x, None, num_groups=4, score="sum", g=torch.zeros(1, 4, 2))


def test_unknown_score_is_rejected():
    x = torch.randn(1, 4, 2, 64)
    with pytest.raises(ValueError, match="score"):
        kata_attn_state(x, x, num_groups=4, score="dot")


def test_state_shape_mismatch_is_rejected():
    with pytest.raises(ValueError):
        kata_attn_state(torch.randn(1, 4, 2, 64), torch.randn(1, 4, 3, 64), num_groups=4)
    with pytest.raises(ValueError):
        kata_attn_state(torch.randn(1, 4, 2, 60), torch.randn(1, 4, 2, 60), num_groups=8)


def test_varlen_rejects_unpacked_inputs_and_bad_totals():
    x = torch.randn(2, 10, 2, 64)
    with pytest.raises(ValueError, match="packed"):
        parallel_kata_attn_varlen(x, x, x, torch.tensor([0, 10]))
    y = torch.randn(1, 10, 2, 64)
    with pytest.raises(ValueError, match="covers"):
        parallel_kata_attn_varlen(y, y, y, torch.tensor([0, 4, 9]))
    with pytest.raises(ValueError, match="score"):
        parallel_kata_attn_varlen(y, y, y, torch.tensor([0, 10]), score="dot")
