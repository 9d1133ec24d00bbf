"""FlexReuseBackend on the GPU: phases, routes and outputs against the oracle.

Mirrors the reference's backend tests (tests/test_flex_route_update.py) at
head_dim 128, plus route parity through the whole phase machine.
"""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from dit_sparse_atten_b200 import _native, kernels
from dit_sparse_atten_b200 import flex as flex_module
from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig
from dit_sparse_atten_b200.spatial import build_spatial_layout
from oracle import attention as oatt
from oracle import route as oroute

pytestmark = pytest.mark.gpu
DEV = "cuda"


def ctx(monkeypatch, layer, step, branch, grid):
    monkeypatch.setattr(flex_module, "routing_context",
                        lambda include_grid=False: (layer, step, branch, grid) if include_grid
                        else (layer, step, branch))


def sdpa(q, k, v):
    return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                          v.transpose(1, 2)).transpose(1, 2)


def inputs(tokens, heads, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn((1, tokens, heads, 128), generator=g).to(torch.bfloat16).to(DEV)
            for _ in range(3)]


def close(a, b, max_abs=2e-2, mean_abs=2e-3):
    d = (a.float() - b.float()).abs()
    assert float(d.max()) <= max_abs and float(d.mean()) <= mean_abs, (float(d.max()),
                                                                       float(d.mean()))


def oracle_sparse(q, k, v, route, layout, block=128):
    """Reference output of the packed route, returned in the original token order."""
    perm = layout.permutation_cpu.numpy() if layout is not None else None
    qn, kn, vn = (x[0].float().cpu().numpy() for x in (q, k, v))
    if perm is not None:
        qn, kn, vn = qn[perm], kn[perm], vn[perm]
    out = oatt.block_sparse_attention(qn, kn, vn, route, block)
    if perm is not None:
        restored = np.empty_like(out)
        restored[perm] = out
        out = restored
    return torch.from_numpy(out)


def test_sampled_bootstrap_reuse_and_update_with_spatial_reorder(monkeypatch):
    grid = (4, 16, 32)                      # 2048 tokens, 16 blocks
    q, k, v = inputs(2048, 4, 0)
    cfg = FlexReuseConfig(bootstrap_mode="sampled", prefetch_sampled_bootstrap=False,
                          prefetch_sampled_update=False, sampled_update_interval=2,
                          route_samples=16, route_persistence=0.5, mass_target=0.95,
                          keep=0.625, spatial_reorder=True, total_steps=5)
    backend = FlexReuseBackend(cfg)
    layout = build_spatial_layout(grid, 128)

    ctx(monkeypatch, 1, 0, 0, grid)
    out0 = backend(q, k, v)
    close(out0, sdpa(q, k, v), 2e-3 * 10, 2e-3)
    state = next(iter(backend.state.values()))
    route0 = state["route"].cpu().numpy()
    # the bootstrap route is the reference rule applied to the GPU sampled mass
    qp, kp, _ = layout.reorder_qkv(q, k, v)
    mass = kernels.sampled_block_mass(qp, kp, 128, 16)[0].cpu().numpy()
    ref_route = oroute.sampled_route(mass, None, 0.5, 0.95, 0.625, grid=grid, block=128)
    np.testing.assert_array_equal(route0, ref_route)
    assert state["frontier"] is not None

    ctx(monkeypatch, 1, 1, 0, grid)
    out1 = backend(q, k, v)
    close(out1.cpu(), oracle_sparse(q, k, v, route0, layout))
    assert backend.phase_counts["sparse_reuse"] == 1

    ctx(monkeypatch, 1, 2, 0, grid)
    out2 = backend(q, k, v)
    state = next(iter(backend.state.values()))
    assert backend.phase_counts["sampled_update"] == 1
    ref_route2 = oroute.sampled_route(mass, route0, 0.5, 0.95, 0.625, grid=grid, block=128)
    if state.get("dense"):
        close(out2, sdpa(q, k, v))
    else:
        np.testing.assert_array_equal(state["route"].cpu().numpy(), ref_route2)
        close(out2.cpu(), oracle_sparse(q, k, v, ref_route2, layout))
    assert state["keep"] == oroute.route_keep(ref_route2)
    _native.check_device_errors()


def test_exact_bootstrap_route(monkeypatch):
    q, k, v = inputs(1024, 2, 1)
    backend = FlexReuseBackend(FlexReuseConfig(mass_target=0.9, keep=0.5))
    ctx(monkeypatch, 3, 0, 1, (2, 16, 32))
    out = backend(q, k, v)
    close(out, sdpa(q, k, v))
    state = next(iter(backend.state.values()))
    # the bootstrap's mass: from the same dense attention pass
    _, _, mass = kernels.dense_attention_block_mass(q, k, v)
    mass = mass[0].cpu().numpy()
    expect = oroute.sampled_route(mass, None, 0.0, 0.9, 0.5, grid=(2, 16, 32), block=128)
    np.testing.assert_array_equal(state["route"].cpu().numpy(), expect)
    assert backend.phase_counts["dense_bootstrap"] == 1
    # exact mass against the oracle
    qf, kf = q[0].double().cpu().numpy(), k[0].double().cpu().numpy()
    s = np.einsum("qhd,khd->hqk", qf, kf) * 128 ** -0.5
    m = s.max(-1, keepdims=True)
    lse = (m + np.log(np.exp(s - m).sum(-1, keepdims=True)))[..., 0]
    np.testing.assert_allclose(mass, oroute.exact_block_mass(qf, kf, lse, 128), atol=2e-3)


def test_periodic_route_update_replaces_block_mask(monkeypatch):
    ctx(monkeypatch, 1, 1, 0, None)
    q, k, v = inputs(256, 2, 2)
    backend = FlexReuseBackend(FlexReuseConfig(keep=0.5, mass_target=0.9, update_interval=2))
    backend.state[(1, 0, 256, 2, 128, q.device, None)] = {
        "route": torch.zeros(2, 2, 2, device=DEV, dtype=torch.bool),
        "block_mask": object(), "step": -1}
    output = backend(q, k, v)
    assert output.shape == q.shape
    state = next(iter(backend.state.values()))
    assert state["step"] == 1
    assert state["route"].any()
    assert isinstance(state["block_mask"], flex_module.BlockRoute)


def test_sampled_update_can_switch_route_to_dense(monkeypatch):
    ctx(monkeypatch, 1, 1, 0, None)
    q, k, v = inputs(256, 2, 3)
    backend = FlexReuseBackend(FlexReuseConfig(sampled_update_interval=1,
                                               prefetch_sampled_update=False,
                                               dense_route_threshold=0.75, total_steps=3))
    backend.install_route(torch.eye(2, dtype=torch.bool).expand(2, 2, 2), attention_id=1,
                          branch=0, tokens=256, heads=2, head_dim=128, device=DEV)
    backend.state[next(iter(backend.state))]["step"] = 0
    ones = kernels.route_select(torch.ones(2, 2, 2, device=DEV), target=1.0, keep=1.0)
    monkeypatch.setattr(backend, "_sampled_route",
                        lambda state, query, key, scale: backend._result_from_csr(state, ones, 256))
    out = backend(q, k, v)
    close(out, sdpa(q, k, v))
    assert backend.state[next(iter(backend.state))]["dense"] is True
    assert backend.phase_counts["dense_dispatch"] == 1


def test_spatial_bootstrap_restores_original_token_order(monkeypatch):
    ctx(monkeypatch, 1, 0, 0, (1, 4, 64))
    q, k, v = inputs(256, 2, 8)
    backend = FlexReuseBackend(FlexReuseConfig(
        bootstrap_mode="sampled", prefetch_sampled_bootstrap=False, spatial_reorder=True,
        spatial_microtile_tokens=32, route_samples=2, total_steps=2))
    out = backend(q, k, v)
    close(out, sdpa(q, k, v), 2e-2, 2e-3)
    state = next(iter(backend.state.values()))
    assert state["layout"].microtile_shape == (4, 8)
    assert state["frontier"] is not None


def test_prefetched_bootstrap_is_activated_next_step(monkeypatch):
    grid = (2, 16, 32)
    q, k, v = inputs(1024, 2, 9)
    backend = FlexReuseBackend(FlexReuseConfig(bootstrap_mode="sampled", route_samples=16,
                                               mass_target=0.9, keep=0.625))
    ctx(monkeypatch, 2, 0, 0, grid)
    backend(q, k, v)
    state = next(iter(backend.state.values()))
    assert "pending" in state and backend.phase_counts["sampled_bootstrap"] == 1
    ctx(monkeypatch, 2, 1, 0, grid)
    out = backend(q, k, v)
    state = next(iter(backend.state.values()))
    assert "pending" not in state and state["route"] is not None
    if not state["dense"]:
        close(out.cpu(), oracle_sparse(q, k, v, state["route"].cpu().numpy(), None))
