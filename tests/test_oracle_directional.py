"""The directional frontier update of the oracle (``oracle/route.py``)
against the reference's own outputs (``tests/golden/directional.npz``) and the
known answers of the reference's tests (tests/test_directional_routing.py:
9-48), bit for bit."""

import numpy as np

from conftest import DIRECTIONAL_KEYS, directional_case, sha256_tensor, unpack_route
from oracle import route as oroute


def line_neighbors(blocks):
    """Neighbours of a 1-D strip: left in slot 2, right in slot 3
    (tests/test_directional_routing.py:9-16)."""
    nb = np.full((blocks, 4), -1, np.int32)
    for b in range(blocks):
        if b:
            nb[b, 2] = b - 1
        if b + 1 < blocks:
            nb[b, 3] = b + 1
    return nb


def test_frontier_kat():
    route = np.zeros((1, 4, 4), bool)
    route[:, :, 1:3] = True
    frontier = oroute.frontier_mask(route, line_neighbors(4))
    assert frontier[:, :, 1:3].all()
    assert not frontier[:, :, [0, 3]].any()


def test_update_kat_replaces_low_score_edge_at_fixed_budget():
    blocks = 4
    route = np.eye(blocks, dtype=bool)[None]
    mass = route.astype(np.float32)
    for row in range(blocks - 1):
        mass[0, row, row + 1] = 2.0
    result = oroute.directional_budget_update(mass, route, line_neighbors(blocks), keep=.5,
                                              persistence=0, expand_q=False, expand_k=True,
                                              expand_joint=False)
    updated = result["route"]
    assert (updated.sum(-1) == 1).all()
    assert updated[0, 0, 1] and updated[0, 1, 2] and updated[0, 2, 3] and updated[0, 3, 3]
    assert result["added"].sum() == 3
    assert result["dropped"].sum() == 3


def test_inputs_match_the_fixture_digests(golden):
    import torch

    masses, _, _, _, g = directional_case(golden)
    for name, mass in masses.items():
        assert sha256_tensor(torch.from_numpy(mass)) == str(g[f"{name}_sha"])


def test_directional_update_matches_reference(golden):
    masses, prev, nb, options, g = directional_case(golden)
    front = oroute.frontier_mask(prev, nb)
    for name, mass in masses.items():
        for i, opts in enumerate(options):
            got = oroute.directional_budget_update(mass, prev, nb, keep=0.625,
                                                   previous_frontier=front, **opts)
            for key in DIRECTIONAL_KEYS:
                want = unpack_route(g[f"{name}{i}_{key}"], 450)
                assert np.array_equal(got[key], want), (name, i, key)
            sunk = oroute.directional_route(mass, prev, nb, grid=(16, 45, 80), block=128,
                                            keep=0.625, previous_frontier=front, **opts)
            assert np.array_equal(sunk["route"], unpack_route(g[f"{name}{i}_sunk_route"], 450))
            assert np.array_equal(sunk["frontier"],
                                  unpack_route(g[f"{name}{i}_sunk_frontier"], 450))


def test_frontier_computed_when_not_given(golden):
    masses, prev, nb, options, g = directional_case(golden)
    got = oroute.directional_budget_update(masses["plain"], prev, nb, keep=0.625, **options[0])
    assert np.array_equal(got["route"], unpack_route(g["plain0_route"], 450))
