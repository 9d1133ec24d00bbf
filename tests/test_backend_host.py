"""Host-side behaviour of the backend mirror (no GPU): config validation, phase
decisions that stay on the dense path, the sink rule and loud failure of the
sparse path on CPU tensors.  Mirrors the reference's own CPU tests
(tests/test_flex_route_update.py:106-132, tests/test_runtime_context.py:63-84).
"""

import pytest
import torch

import dit_sparse_atten_b200 as bsa
from dit_sparse_atten_b200 import flex as flex_module
from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig


@pytest.mark.parametrize("kwargs,message", [
    ({"block_size": 64}, "128-token blocks"),
    ({"update_interval": -1}, "update_interval"),
    ({"sampled_update_interval": -2}, "sampled_update_interval"),
    ({"update_interval": 1, "sampled_update_interval": 1}, "mutually exclusive"),
    ({"route_samples": 0}, "route_samples"),
    ({"route_persistence": -1.0}, "route_persistence"),
    ({"bootstrap_mode": "dense"}, "bootstrap_mode"),
    ({"dense_route_threshold": 0.0}, "dense_route_threshold"),
    ({"keep": 1.5}, "keep"),
    ({"mass_target": 0.0}, "mass_target"),
    ({"spatial_microtile_tokens": 0}, "spatial_microtile_tokens"),
    ({"route_budget_scale": 0.0}, "route_budget_scale"),
    ({"route_exploration_fraction": 2.0}, "route_exploration_fraction"),
    ({"directional_update": True}, "requires spatial_reorder"),
])
def test_config_validation_matches_reference(kwargs, message):
    with pytest.raises(ValueError, match=message):
        FlexReuseBackend(FlexReuseConfig(**kwargs))


def test_directional_update_config_is_accepted():
    backend = FlexReuseBackend(FlexReuseConfig(directional_update=True, spatial_reorder=True,
                                               route_exploration_fraction=0.1))
    assert backend.config.directional_update


def test_directional_update_fails_loudly_on_cpu():
    from dit_sparse_atten_b200 import routing

    mass = torch.rand(1, 4, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        routing.directional_budget_update(mass, mass > 0.5, torch.full((4, 4), -1), keep=0.5)
    with pytest.raises(ValueError, match="identical shapes"):
        routing.directional_budget_update(mass, mass[0] > 0.5, torch.full((4, 4), -1), keep=0.5)
    with pytest.raises(ValueError, match=r"neighbors must have shape \[blocks, 4\]"):
        routing.directional_budget_update(mass, mass > 0.5, torch.full((3, 4), -1), keep=0.5)


def test_first_frame_sink_is_added_to_every_query_row():
    backend = FlexReuseBackend(FlexReuseConfig(block_size=128))
    route = torch.zeros(2, 4, 4, dtype=torch.bool)
    result = backend._add_first_frame_sink({"grid": (2, 8, 16), "layout": None}, {"route": route})
    assert result["route"][..., 0].all()
    assert not result["route"][..., 1:].any()
    assert backend._sink_blocks({"grid": (16, 45, 80)}) == 29
    assert backend._sink_blocks({"grid": (21, 30, 52)}) == 13


def test_first_layer_is_always_dense(monkeypatch):
    monkeypatch.setattr(flex_module, "routing_context",
                        lambda include_grid=False: (0, 3, 1, (2, 2, 2)) if include_grid
                        else (0, 3, 1))
    q = torch.randn(1, 8, 2, 4)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    backend = FlexReuseBackend()
    output = backend(q, k, v, dtype=torch.float32)
    reference = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    torch.testing.assert_close(output, reference)
    assert backend.state == {}
    assert backend.phase_counts["first_layer_dense"] == 1


def test_unsupported_modes_fall_back_to_dense():
    backend = FlexReuseBackend()
    q = torch.randn(2, 8, 2, 4)  # batch 2, as the reference's dense fallback
    out = backend(q, q, q, dtype=torch.float32)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2), q.transpose(1, 2), q.transpose(1, 2)).transpose(1, 2)
    torch.testing.assert_close(out, ref)


def test_sparse_path_fails_loudly_on_cpu(monkeypatch):
    monkeypatch.setattr(flex_module, "routing_context",
                        lambda include_grid=False: (1, 1, 0, None) if include_grid else (1, 1, 0))
    backend = FlexReuseBackend(FlexReuseConfig(bootstrap_mode="sampled",
                                               prefetch_sampled_bootstrap=False))
    q = torch.randn(1, 256, 2, 128)
    route = torch.ones(2, 2, 2, dtype=torch.bool)
    csr = flex_module.BlockRoute(route.sum(-1, dtype=torch.int32)[None],
                                 torch.arange(2, dtype=torch.int32).expand(1, 2, 2, 2), 256, 128)
    backend.state[(1, 0, 256, 2, 128, q.device, None)] = {
        "route": route, "block_mask": csr, "step": 0, "dense": False}
    with pytest.raises(RuntimeError, match="CUDA"):
        backend(q, q, q)


def test_routing_context_roundtrip():
    bsa.reset_runtime_state()
    assert bsa.routing_context(include_grid=True) == (-1, -1, -1, None)
    bsa.set_routing_context(attention_id=3, step=2, branch=1, grid=(16, 45, 80))
    assert bsa.routing_context() == (3, 2, 1)
    assert bsa.routing_context(include_grid=True)[3] == (16, 45, 80)
    bsa.reset_runtime_state()


def test_custom_context_provider_is_used():
    calls = []

    def provider(include_grid=False):
        calls.append(include_grid)
        return (0, 0, 0, None)

    backend = FlexReuseBackend(routing_context=provider)
    q = torch.randn(1, 8, 2, 4)
    backend(q, q, q, dtype=torch.float32)
    assert calls == [True]


def test_registry():
    assert isinstance(bsa.get_backend("dense"), bsa.DenseBackend)
    backend = bsa.get_backend("flex_reuse", keep=0.5, bootstrap_mode="sampled")
    assert backend.config.keep == 0.5
    with pytest.raises(ValueError):
        bsa.get_backend("sparse")


def test_keep_cap_matches_python_ceil():
    from dit_sparse_atten_b200.kernels import keep_cap
    import math
    for cols in (1, 5, 256, 450, 1000):
        for keep in (0.58, 0.625, 0.3, 1.0, 1e-9):
            assert keep_cap(cols, keep) == max(1, math.ceil(cols * keep))


def test_profile_summary_shape():
    backend = FlexReuseBackend()
    summary = backend.profile_summary()
    assert set(summary) == {"phase_counts", "active_routes", "released_routes",
                            "mean_route_keep", "mean_frontier_fraction",
                            "dense_dispatched_routes"}


def _sdpa(q, k, v):
    return torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)


def test_sampled_update_can_switch_route_to_dense_on_cpu(monkeypatch):
    """The reference's CPU test (tests/test_flex_route_update.py:41-73): an
    injected dict state, a substituted route producer returning a dict, and
    the dense switch at keep >= threshold, all without a GPU."""
    monkeypatch.setattr(flex_module, "routing_context",
                        lambda include_grid=False: (1, 1, 0, None) if include_grid
                        else (1, 1, 0))
    monkeypatch.setattr(flex_module, "_build_block_mask", lambda *args: object())
    q = torch.randn(1, 8, 1, 4)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    backend = FlexReuseBackend(FlexReuseConfig(sampled_update_interval=1,
                                               prefetch_sampled_update=False,
                                               dense_route_threshold=.75, total_steps=3))
    backend.state[(1, 0, 8, 1, 4, q.device, None)] = {
        "route": torch.eye(1, dtype=torch.bool), "block_mask": object(), "step": 0,
        "dense": False}
    monkeypatch.setattr(backend, "_sampled_route",
                        lambda state, query, key, scale: {
                            "route": torch.ones(1, 1, 1, dtype=torch.bool), "frontier": None})
    output = backend(q, k, v, dtype=torch.float32)
    torch.testing.assert_close(output, _sdpa(q, k, v))
    state = backend.state[next(iter(backend.state))]
    assert state["dense"] is True
    assert state["route"] is None and state["block_mask"] is None
    assert state["keep"] == 1.0 and state["step"] == 1
    assert backend.phase_counts["dense_dispatch"] == 1
    assert backend.phase_counts["sampled_update"] == 1
    assert "pending" not in state


def test_dense_state_is_released_at_the_final_step(monkeypatch):
    """A dense-dispatched route keeps answering with SDPA and is released at
    the last step; the summary counts it among the released routes."""
    step = {"value": 1}
    monkeypatch.setattr(flex_module, "routing_context",
                        lambda include_grid=False: (2, step["value"], 1, None))
    q = torch.randn(1, 8, 2, 4)
    backend = FlexReuseBackend(FlexReuseConfig(total_steps=3, dense_route_threshold=0.5))
    backend.state[(2, 1, 8, 2, 4, q.device, None)] = {"dense": True, "keep": 0.8, "step": 0}
    torch.testing.assert_close(backend(q, q, q, dtype=torch.float32), _sdpa(q, q, q))
    assert len(backend.state) == 1
    step["value"] = 2
    torch.testing.assert_close(backend(q, q, q, dtype=torch.float32), _sdpa(q, q, q))
    assert backend.state == {}
    summary = backend.profile_summary()
    assert summary["phase_counts"]["dense_dispatch"] == 2
    assert summary["released_routes"] == 1 and summary["active_routes"] == 0
    assert summary["dense_dispatched_routes"] == 1
    assert summary["mean_route_keep"] == 0.8
    assert backend.finished_routes == [{"keep": 0.8, "frontier_fraction": None, "dense": True}]
