"""CPU: the in_proj deal of the persistent decode kernel (lssm_persist_in_deal, the function the
kernel itself calls): every channel unit and every B / C / dt tile goes to exactly one CTA, the
units of a CTA are contiguous (its state rows are one range), and a CTA holding a B / C / dt
tile, which runs as a group of its own, is charged two units so the busiest CTAs are not the
ones that also publish the rows every CTA polls."""

import ctypes as C
import itertools

import pytest

import lssm


def deal(G, di, nspec):
    out = (C.c_uint32 * 4)()
    rows = []
    for s in range(G):
        lssm.lib().lssm_persist_in_deal(s, G, di, nspec, out)
        rows.append(tuple(out))
    return rows   # (first unit, units, first special tile, special tiles)


@pytest.mark.parametrize("G,di,nspec", list(itertools.product([148, 132, 16, 8], [5120, 4096, 2560, 1536, 768, 256],
                                                              [21, 5, 1, 40, 200])))
def test_every_unit_and_tile_dealt_once(G, di, nspec):
    rows = deal(G, di, nspec)
    pos = 0
    for ub, nu, _, _ in rows:
        assert ub == pos, "units of consecutive CTAs must be contiguous"
        pos += nu
    assert pos == di // 8
    tiles = sorted(kf + i * G for _, _, kf, nsp in rows for i in range(nsp))
    assert tiles == list(range(nspec))


def test_2p7b_shape_charges_special_tiles_two_units():
    """2.7B: 640 units and 21 B / C / dt tiles on 148 SMs. The 21 CTAs with a special tile take
    3 units; the rest take 5 or 4, so no CTA runs more than 5 tile-equivalents."""
    rows = deal(148, 5120, 21)
    shape = {}
    for _, nu, _, nsp in rows:
        shape[(nu, nsp)] = shape.get((nu, nsp), 0) + 1
    assert shape == {(3, 1): 21, (5, 0): 69, (4, 0): 58}
    assert max(nu + 2 * nsp for _, nu, _, nsp in rows) == 5


@pytest.mark.parametrize("G,di,nspec", [(148, 5120, 21), (132, 5120, 21), (148, 4096, 40), (148, 8192, 40)])
def test_charged_deal_is_balanced(G, di, nspec):
    """Where the charged deal applies, every CTA's cost (units + 2 per special tile) is within one
    of the ceiling of the average."""
    rows = deal(G, di, nspec)
    T = -(-(di // 8 + 2 * nspec) // G)
    costs = [nu + 2 * nsp for _, nu, _, nsp in rows]
    assert max(costs) == T and min(costs) >= T - 2
