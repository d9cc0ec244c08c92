"""Head groups of flashmlp_b200.host.HostPipeline (no GPU): every head exactly once, in
order, with smaller groups at both ends of the pipeline when there is room for them."""
import pytest

from flashmlp_b200.host import HostPipeline


def groups(H, hg, ramp=True):
    p = object.__new__(HostPipeline)  # _groups needs no device
    p.ramp = ramp
    return [b - a for a, b in p._groups(H, hg)], p._groups(H, hg)


@pytest.mark.parametrize("H,hg", [(32, 4), (16, 2), (4, 1), (8, 4), (12, 4), (33, 4), (13, 4), (1, 4), (9, 3)])
@pytest.mark.parametrize("ramp", [True, False])
def test_groups_cover_every_head_in_order(H, hg, ramp):
    sizes, ranges = groups(H, hg, ramp)
    assert sum(sizes) == H and all(s >= 1 for s in sizes) and max(sizes) <= max(hg, 1)
    assert ranges[0][0] == 0 and ranges[-1][1] == H
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(len(ranges) - 1))


def test_ramp_shapes():
    assert groups(32, 4)[0] == [1, 2, 4, 4, 4, 4, 4, 4, 2, 2, 1]
    assert groups(32, 4, ramp=False)[0] == [4] * 8
    assert groups(8, 4)[0] == [4, 4]  # no room for the ramp
    assert groups(4, 1)[0] == [1, 1, 1, 1]
