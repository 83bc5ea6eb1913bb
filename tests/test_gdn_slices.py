"""Host logic of the gated delta rule's value slicing (no GPU): value heads wider than the kernels'
64 columns run as independent slices of the state that together cover the head exactly once."""

from __future__ import annotations

from linatt_b200.gated_delta_rule import KDIM, _value_slices


def test_value_slices_cover_the_head_once():
    assert _value_slices(KDIM) == [(0, KDIM)]
    assert _value_slices(40) == [(0, 40)]
    for V in (65, 96, 128, 200, 256):
        sl = _value_slices(V)
        assert sl[0][0] == 0 and sl[-1][1] == V
        assert all(b - a <= KDIM and a < b for a, b in sl)
        assert all(sl[i][1] == sl[i + 1][0] for i in range(len(sl) - 1))
