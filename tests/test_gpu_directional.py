"""GPU parity of the directional frontier update (``csrc/directional.cu``)
through the C ABI: against the reference's own outputs
(``tests/golden/directional.npz``), the reference tests' known answers
(tests/test_directional_routing.py:19-48) and the oracle on random cases with
ties, ragged block counts, missing neighbours and several planes.  Index work:
bit-exact everywhere.
"""

import numpy as np
import pytest
import torch

from conftest import DIRECTIONAL_KEYS, directional_case, unpack_route
from dit_sparse_atten_b200 import _native, kernels, routing
from dit_sparse_atten_b200 import flex as flex_module
from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig
from dit_sparse_atten_b200.spatial import build_spatial_layout
from oracle import route as oroute

pytestmark = pytest.mark.gpu
DEV = "cuda"


def line_neighbors(blocks):
    nb = torch.full((blocks, 4), -1, dtype=torch.int32)
    for b in range(blocks):
        if b:
            nb[b, 2] = b - 1
        if b + 1 < blocks:
            nb[b, 3] = b + 1
    return nb


def gpu(x):
    return torch.as_tensor(x).to(DEV)


def assert_same(got, want, what):
    got = got.cpu().numpy() if isinstance(got, torch.Tensor) else got
    assert np.array_equal(got, want), (what, int((got != want).sum()))


def check_against_oracle(mass, prev, nb, sink_blocks=0, front=None, **opts):
    """All outputs of one GPU call against the oracle, CSR and kept included."""
    keep = opts.pop("keep", 0.625)
    r = kernels.directional_update(gpu(mass), gpu(prev), gpu(nb), keep=keep,
                                   previous_frontier=None if front is None else gpu(front),
                                   sink_blocks=sink_blocks, **opts)
    torch.cuda.synchronize()
    _native.check_device_errors()
    ref = oroute.directional_budget_update(mass, prev, nb, keep=keep, previous_frontier=front,
                                           **opts)
    for key in ("candidates", "exploration", "dropped", "added"):
        assert_same(getattr(r, key), ref[key], key)
    sunk = ref["route"].copy()
    sunk[..., :sink_blocks] = True
    assert_same(r.route, sunk, "route")
    assert_same(r.frontier, oroute.frontier_mask(sunk, nb), "frontier")
    counts, indices = oroute.pack_boolean_rows(sunk)
    assert_same(r.counts, counts, "counts")
    assert_same(r.indices, indices, "indices")
    assert_same(r.kept, sunk.reshape(-1, sunk.shape[-1] ** 2).sum(-1), "kept")
    return r


def test_frontier_kat():
    route = torch.zeros(1, 4, 4, dtype=torch.bool)
    route[:, :, 1:3] = True
    frontier = routing.frontier_mask(gpu(route), line_neighbors(4)).cpu()
    assert frontier[:, :, 1:3].all()
    assert not frontier[:, :, [0, 3]].any()


def test_update_kat_replaces_low_score_edge_at_fixed_budget():
    blocks = 4
    route = torch.eye(blocks, dtype=torch.bool).unsqueeze(0)
    mass = route.float()
    for row in range(blocks - 1):
        mass[0, row, row + 1] = 2.0
    result = routing.directional_budget_update(
        gpu(mass), gpu(route), line_neighbors(blocks), keep=.5, persistence=0,
        expand_q=False, expand_k=True, expand_joint=False)
    updated = result["route"].cpu()
    assert (updated.sum(-1) == 1).all()
    assert updated[0, 0, 1] and updated[0, 1, 2] and updated[0, 2, 3] and updated[0, 3, 3]
    assert int(result["added"].sum()) == 3
    assert int(result["dropped"].sum()) == 3


@pytest.mark.parametrize("mass_name", ["plain", "quant"])
def test_matches_reference_fixtures(golden, mass_name):
    masses, prev, nb, options, g = directional_case(golden)
    mass = masses[mass_name]
    front = oroute.frontier_mask(prev, nb)
    for i, opts in enumerate(options):
        got = routing.directional_budget_update(gpu(mass), gpu(prev), gpu(nb), keep=0.625,
                                                previous_frontier=gpu(front), **opts)
        for key in DIRECTIONAL_KEYS:
            assert_same(got[key], unpack_route(g[f"{mass_name}{i}_{key}"], 450), (i, key))
        # the backend's fused call: sink (29 blocks at 720p) and frontier of the sunk route
        r = kernels.directional_update(gpu(mass), gpu(prev), gpu(nb), keep=0.625,
                                       previous_frontier=None, sink_blocks=29, **opts)
        assert_same(r.route, unpack_route(g[f"{mass_name}{i}_sunk_route"], 450), (i, "sunk"))
        assert_same(r.frontier, unpack_route(g[f"{mass_name}{i}_sunk_frontier"], 450),
                    (i, "sunk frontier"))
    _native.check_device_errors()


def random_case(planes, blocks, seed, quantise, missing=0.15):
    rng = np.random.default_rng(seed)
    mass = rng.random((*planes, blocks, blocks), dtype=np.float32) ** 4
    mass = (mass / mass.sum(-1, keepdims=True)).astype(np.float32)
    if quantise:
        mass = (np.round(mass * np.float32(blocks * 16)) / np.float32(blocks * 16)).astype(np.float32)
    prev = rng.random(mass.shape) < 0.3
    nb = rng.integers(0, blocks, size=(blocks, 4)).astype(np.int32)
    nb[rng.random((blocks, 4)) < missing] = -1
    return mass, prev, nb


@pytest.mark.parametrize("planes,blocks,seed", [
    ((1,), 1, 0), ((2,), 5, 1), ((2, 3), 37, 2), ((1, 2), 129, 3), ((4,), 450, 4)])
@pytest.mark.parametrize("quantise", [False, True])
def test_random_cases_match_oracle(planes, blocks, seed, quantise):
    mass, prev, nb = random_case(planes, blocks, seed, quantise)
    sink = min(3, blocks)
    for opts in ({}, {"min_ratio": 0.8, "candidate_bonus": 0.5, "budget_scale": 1.3,
                      "exploration_fraction": 0.1},
                 {"persistence": 0.0, "expand_q": False, "exploration_fraction": 1.0},
                 {"expand_q": False, "expand_k": False, "budget_scale": 0.5}):
        check_against_oracle(mass, prev, nb, sink_blocks=sink, **opts)
        check_against_oracle(mass, prev, nb, front=oroute.frontier_mask(prev, nb), **opts)


def test_wide_rows_use_large_shared_memory():
    """2,100 blocks per row: 4,096-entry sort keys, > 48 KB of shared memory."""
    mass, prev, nb = random_case((1,), 2100, 5, True, missing=0.05)
    check_against_oracle(mass, prev, nb, sink_blocks=13, exploration_fraction=0.01)


def test_frontier_matches_oracle_on_random_routes():
    rng = np.random.default_rng(6)
    for planes, blocks in (((3,), 37), ((2, 2), 450)):
        route = rng.random((*planes, blocks, blocks)) < 0.4
        nb = rng.integers(-1, blocks, size=(blocks, 4)).astype(np.int32)
        got = kernels.frontier_mask(gpu(route), gpu(nb))
        assert_same(got, oroute.frontier_mask(route, nb), "frontier")


def test_out_of_range_neighbor_is_reported():
    route = torch.ones(1, 4, 4, dtype=torch.bool, device=DEV)
    nb = line_neighbors(4)
    nb[1, 0] = 9
    kernels.frontier_mask(route, nb)
    with pytest.raises(RuntimeError, match="out of range"):
        _native.check_device_errors()


def test_backend_sampled_update_uses_directional_route(monkeypatch):
    grid = (4, 16, 32)                      # 2048 tokens, 16 blocks
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn((1, 2048, 4, 128), generator=g).to(torch.bfloat16).to(DEV)
               for _ in range(3))
    cfg = FlexReuseConfig(bootstrap_mode="sampled", prefetch_sampled_bootstrap=False,
                          prefetch_sampled_update=False, sampled_update_interval=2,
                          route_samples=16, route_persistence=0.5, mass_target=0.95, keep=0.625,
                          spatial_reorder=True, directional_update=True,
                          route_exploration_fraction=0.1, direction_candidate_bonus=0.2,
                          total_steps=5)
    backend = FlexReuseBackend(cfg)
    layout = build_spatial_layout(grid, 128)

    def ctx(step):
        monkeypatch.setattr(flex_module, "routing_context",
                            lambda include_grid=False: (1, step, 0, grid) if include_grid
                            else (1, step, 0))

    ctx(0)
    backend(q, k, v)
    state = next(iter(backend.state.values()))
    route0 = state["route"].cpu().numpy()
    front0 = state["frontier"].cpu().numpy()
    qp, kp, _ = layout.reorder_qkv(q, k, v)
    mass = kernels.sampled_block_mass(qp, kp, 128, 16)[0].cpu().numpy()
    nb = layout.neighbors_cpu.numpy()
    np.testing.assert_array_equal(front0, oroute.frontier_mask(route0, nb))
    ctx(1)
    backend(q, k, v)
    ctx(2)
    backend(q, k, v)
    assert backend.phase_counts["sampled_update"] == 1
    state = next(iter(backend.state.values()))
    expect = oroute.directional_route(
        mass, route0, nb, grid=grid, block=128, keep=0.625, persistence=0.5,
        candidate_bonus=0.2, exploration_fraction=0.1, previous_frontier=front0)
    if not state.get("dense"):
        np.testing.assert_array_equal(state["route"].cpu().numpy(), expect["route"])
        np.testing.assert_array_equal(state["frontier"].cpu().numpy(), expect["frontier"])
    assert state["keep"] == oroute.route_keep(expect["route"])
    _native.check_device_errors()
