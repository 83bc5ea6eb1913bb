"""Host-side packing of the varlen API (no kernels): documents scattered into zero-padded rows
and gathered back, with the gradient of the round trip, and rejection of bad cu_seqlens."""

import pytest
import torch

from linatt_b200.varlen import pack_rows, unpack_rows, varlen_index


def test_pack_unpack_round_trip_and_layout():
    cu = torch.tensor([0, 5, 5, 12, 13])  # includes an empty document
    x = torch.randn(1, 13, 2, 3, requires_grad=True)
    dst, N, T_max = varlen_index(cu)
    assert (N, T_max) == (4, 7)
    p = pack_rows(x, dst, N, T_max)
    assert p.shape == (4, 7, 2, 3)
    assert torch.equal(p[0, :5], x[0, :5]) and torch.equal(p[2, :7], x[0, 5:12]) and torch.equal(p[3, 0], x[0, 12])
    assert torch.count_nonzero(p[0, 5:]) == 0 and torch.count_nonzero(p[1]) == 0 and torch.count_nonzero(p[3, 1:]) == 0
    y = unpack_rows(p, dst)
    assert torch.equal(y, x)
    g = torch.randn_like(y)
    y.backward(g)
    assert torch.equal(x.grad, g)


def test_varlen_index_with_given_max_and_total_matches():
    cu = torch.tensor([0, 3, 10, 11])
    a = varlen_index(cu)
    b = varlen_index(cu, max_seqlen=7, total=11)
    assert torch.equal(a[0], b[0]) and a[1:] == b[1:]


@pytest.mark.parametrize("cu", [[1, 4], [0, 5, 3], [0]])
def test_varlen_index_rejects_bad_cu_seqlens(cu):
    with pytest.raises(ValueError):
        varlen_index(torch.tensor(cu))


@pytest.mark.parametrize("cu,max_seqlen,msg", [([0, 3, 10], 5, "below the longest"), ([0, 3, 9], 7, "covers"),
                                               ([0, 4, 2, 10], 8, "non-decreasing")])
def test_varlen_api_checks_host_cu_seqlens_even_with_max_seqlen(cu, max_seqlen, msg):
    from linatt_b200.varlen import parallel_kata_attn_varlen

    q = torch.zeros(1, 10, 1, 64)
    with pytest.raises(ValueError, match=msg):
        parallel_kata_attn_varlen(q, q, q, torch.tensor(cu), max_seqlen=max_seqlen)
