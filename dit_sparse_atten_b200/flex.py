"""``flex_reuse`` attention backend on the B200 kernels of ``libbsa.so``.

Drop-in for ``attention_backends/flex.py`` of the reference study: the same
``FlexReuseConfig`` fields and validation (``flex.py:43-80,407-443``), the same
callable signature (``flex.py:636-651``) and phase machine (layer-0 dense,
step-0 dense output with an exact or sampled route bootstrap, route reuse,
exact refresh or sampled update, dense dispatch at a keep threshold, release
at the final step; ``flex.py:652-850``), and the same module-level helpers
(``_sampled_block_mass``, ``_top_mass_route``, ``_pack_route``,
``_build_block_mask``, ``_flex_output``, ``_block_attention_mass``,
``_dense_bootstrap``).  What changes is underneath: FlexAttention, the Triton
kernels and the PyTorch route arithmetic are replaced by the sm_100a kernels
(block-sparse attention, sampled/exact block mass, fused prior + top-mass +
sink + CSR selection, directional frontier update, row gather).  The sparse
path needs CUDA bf16 tensors with head_dim 128 and raises otherwise.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, fields
from typing import NamedTuple

import numpy as np
import torch

from . import kernels
from .context import routing_context
from .dense import DenseBackend
from .routing import frontier_mask
from .spatial import build_spatial_layout


@dataclass(frozen=True)
class FlexReuseConfig:
    block_size: int = 128
    keep: float = 0.625
    mass_target: float = 0.90
    compile_kernel: bool = True          # accepted for compatibility; nothing is compiled
    update_interval: int = 0
    sampled_update_interval: int = 0
    route_samples: int = 2
    sample_query_block_chunk: int = 16   # accepted; the mass kernel needs no chunking
    route_persistence: float = 0.5
    prefetch_sampled_update: bool = True
    prefetch_sampled_bootstrap: bool = True
    total_steps: int | None = None
    bootstrap_mode: str = "exact"
    dense_route_threshold: float | None = None
    release_after_final_step: bool = True
    spatial_reorder: bool = False
    spatial_microtile_tokens: int = 32
    directional_update: bool = False
    direction_min_ratio: float = 0.0
    direction_candidate_bonus: float = 0.0
    route_budget_scale: float = 1.0
    route_exploration_fraction: float = 0.0
    direction_expand_q: bool = True
    direction_expand_k: bool = True
    direction_expand_joint: bool = True
    first_frame_sink: bool = True
    first_layer_dense: bool = True


# ----------------------------------------------------------------------------
# Module-level helpers with the reference's names and argument meaning.
# ----------------------------------------------------------------------------

def _top_mass_route(mass, target, keep):
    """Boolean route from block mass ``[..., Q, K]`` (``flex.py:83-94``)."""
    result = kernels.route_select(mass.float(), target=target, keep=keep, want_csr=False,
                                  want_kept=False)
    return result.route.bool()


def _sampled_block_mass(q, k, block_size, samples=2, scale=None, query_block_chunk=16):
    """Sampled block mass ``[H, Qb, Kb]`` for batch-1 ``[1, T, H, D]`` (``flex.py:205-251``)."""
    if q.shape[0] != 1 or q.shape[1] != k.shape[1]:
        raise ValueError("sampled route update supports batch-1 self-attention")
    if samples <= 0 or samples > block_size:
        raise ValueError("route_samples must be in [1, block_size]")
    if query_block_chunk <= 0:
        raise ValueError("sample_query_block_chunk must be positive")
    return kernels.sampled_block_mass(q.to(torch.bfloat16), k.to(torch.bfloat16), block_size,
                                      samples, scale)[0]


def _block_attention_mass(q, k, lse=None, block_size=128, scale=None):
    """Exact dense block mass ``[H, Qb, Kb]`` (``flex.py:167-202``).

    ``lse`` ``[1, H, T]`` (or ``[H, T]``) is the dense pass's per-query
    log-sum-exp, as in the reference; without it the kernel computes it in a
    first pass over the keys.
    """
    if q.shape[0] != 1 or q.shape[1] != k.shape[1]:
        raise ValueError("Flex bootstrap supports batch-1 self-attention")
    if lse is not None and lse.dim() == 2:
        lse = lse.unsqueeze(0)
    return kernels.exact_block_mass(q, k, block_size, scale, lse=lse)[0]


def _pack_route(route):
    """Counts ``[1, H, Q]`` and compact ids ``[1, H, Q, K]`` (``flex.py:275-281``)."""
    counts, indices = kernels.pack_boolean_rows(route)
    return counts.unsqueeze(0), indices.unsqueeze(0)


@dataclass
class BlockRoute:
    """CSR route consumed by the attention kernel (replaces FlexAttention's BlockMask)."""
    counts: torch.Tensor      # int32 [1, H, Qb]
    indices: torch.Tensor     # int32 [1, H, Qb, Kb]: selected ids first
    tokens: int
    block_size: int


def _build_block_mask(route, tokens, block_size):
    """CSR route from a boolean ``[H, Q, K]`` route (``flex.py:308-355``).

    Partial final blocks need no element mask here: the kernel masks keys
    ``>= tokens`` itself and never writes padded query rows.
    """
    if route.dim() != 3 or route.shape[-2] != route.shape[-1]:
        raise ValueError("route must have shape [head, Q-block, K-block]")
    counts, indices = _pack_route(route)
    return BlockRoute(counts, indices, tokens, block_size)


def _flex_output(q, k, v, block_mask, block_size, compile_kernel=True, scale=None,
                 out_rows=None):
    """Block-sparse attention of ``[B, T, H, D]`` tensors over a CSR route.

    With ``out_rows`` (the spatial layout's permutation) the output rows are
    stored straight back to raster order (the unpack folded into the store).
    """
    del compile_kernel
    counts = block_mask.counts
    indices = block_mask.indices
    if counts.dim() == 3 and counts.shape[0] == 1:
        counts, indices = counts[0], indices[0]
    return kernels.block_sparse_attention(q, k, v, counts, indices, block=block_size, scale=scale,
                                          out_rows=out_rows)


def _dense_and_mass(q, k, v, block_size, scale=None):
    """Dense output and exact block mass ``[1, H, Qb, Qb]`` from one attention
    pass (the reference's dense FlexAttention with ``return_lse`` followed by
    ``_block_attention_mass``, ``flex.py:254-272``).  ``(None, None)`` for
    inputs that kernel does not take (not CUDA bf16, D != 128, block != 128)."""
    if (q.dtype != torch.bfloat16 or q.shape[-1] != kernels.HEAD_DIM or not q.is_cuda
            or block_size != 128):
        return None, None
    out, _, mass = kernels.dense_attention_block_mass(q, k, v, scale=scale)
    return out, mass


def _dense_bootstrap(q, k, v, block_size, mass_target, keep, compile_kernel, scale=None):
    """Dense output and its exact block top-mass route (``flex.py:254-272``),
    from one attention pass that also yields the block mass."""
    if q.shape[0] != 1 or q.shape[1] != k.shape[1]:
        raise ValueError("Flex bootstrap supports batch-1 self-attention")
    del compile_kernel
    output, mass = _dense_and_mass(q, k, v, block_size, scale)
    if output is None:
        output = DenseBackend()(q, k, v, softmax_scale=scale, dtype=q.dtype)
        mass = _block_attention_mass(q, k, None, block_size, scale=scale)
    else:
        mass = mass[0]
    return output, _top_mass_route(mass, mass_target, keep)


def _fp32_mean_of_count(count, numel):
    """``float(route.float().mean())`` from an exact integer count."""
    return float(np.float32(np.float32(count) / np.float32(numel)))


# ----------------------------------------------------------------------------
# Backend state: one RouteState per (layer, branch, shape, device, layout) key,
# and a PhaseLog of what the backend did.
# ----------------------------------------------------------------------------

PHASES = ("dense_bootstrap", "sampled_bootstrap", "exact_refresh", "sampled_update",
          "sparse_reuse", "dense_dispatch", "first_layer_dense")


class RouteResult(NamedTuple):
    """A freshly chosen route: bool route, its frontier (or None), per-plane
    kept counts (int64, or None) and the CSR the attention kernel reads."""
    route: torch.Tensor
    frontier: torch.Tensor | None
    kept: torch.Tensor | None
    block_mask: "BlockRoute"


class PendingRoute(NamedTuple):
    """A route computed on the side stream, adopted at the next call."""
    result: RouteResult
    source_step: int
    ready: torch.cuda.Event


@dataclass
class RouteState:
    """Reusable route of one layer and CFG branch.

    Item access (``state["route"]``, ``state.get("dense")``, ``"pending" in
    state``) is kept because the reference exposes its per-route state as
    plain dicts that callers and tests read and inject (``backend.state``).
    """
    route: torch.Tensor | None = None
    frontier: torch.Tensor | None = None
    block_mask: object = None
    kept: torch.Tensor | None = None
    step: int = 0
    layout: object = None
    grid: tuple | None = None
    keep: float | None = None
    frontier_fraction: float | None = None
    dense: bool = False
    pending: PendingRoute | None = None

    @classmethod
    def coerce(cls, value):
        if isinstance(value, cls):
            return value
        names = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in dict(value).items() if k in names})

    def adopt(self, result: RouteResult, step: int | None = None):
        self.route, self.frontier, self.kept, self.block_mask = result
        if step is not None:
            self.step = step

    def drop_route(self):
        self.route = self.frontier = self.kept = self.block_mask = None

    # mapping view ---------------------------------------------------------
    def __contains__(self, name):
        return name in _STATE_FIELDS and not (name == "pending" and self.pending is None)

    def __getitem__(self, name):
        if name not in self:
            raise KeyError(name)
        return getattr(self, name)

    def __setitem__(self, name, value):
        if name not in _STATE_FIELDS:
            raise KeyError(name)
        setattr(self, name, value)

    def get(self, name, default=None):
        return getattr(self, name) if name in self else default


_STATE_FIELDS = frozenset(f.name for f in fields(RouteState))


class ReleasedRoute(NamedTuple):
    keep: float | None
    frontier_fraction: float | None
    dense: bool


class PhaseLog:
    """How often each phase ran, and the keep statistics of released routes."""

    def __init__(self):
        self.counts = dict.fromkeys(PHASES, 0)
        self.released: list[ReleasedRoute] = []

    def hit(self, phase: str):
        self.counts[phase] += 1

    def release(self, state: RouteState):
        self.released.append(ReleasedRoute(state.keep, state.frontier_fraction, bool(state.dense)))

    def summary(self, live) -> dict:
        """The reference's ``profile_summary`` fields (written by its
        ``infer.py:_write_timing``) over live and released routes."""
        live = list(live)
        routed = [s for s in live if s.route is not None]

        def mean(values):
            values = [x for x in values if x is not None]
            return sum(values) / len(values) if values else None

        return {
            "phase_counts": dict(self.counts),
            "active_routes": len(routed),
            "released_routes": len(self.released),
            "mean_route_keep": mean([s.keep for s in routed] + [r.keep for r in self.released]),
            "mean_frontier_fraction": mean([s.frontier_fraction for s in routed]
                                           + [r.frontier_fraction for r in self.released]),
            "dense_dispatched_routes": sum(bool(s.dense) for s in live)
            + sum(r.dense for r in self.released),
        }


class _StateTable(dict):
    """``backend.state``: RouteState values; plain dicts stored by a caller are
    converted on the way in."""

    def __setitem__(self, key, value):
        super().__setitem__(key, RouteState.coerce(value))

    def update(self, *args, **kw):
        for key, value in dict(*args, **kw).items():
            self[key] = value

    def setdefault(self, key, default=None):
        if key not in self:
            self[key] = default if default is not None else RouteState()
        return self[key]


def _validate(c: "FlexReuseConfig"):
    """Construction-time checks; messages follow the reference (``flex.py:408-443``)."""
    checks = (
        (c.block_size == 128,
         "The minimal flex_reuse backend currently supports only 128-token blocks"),
        (c.update_interval >= 0, "update_interval must be zero or a positive integer"),
        (c.sampled_update_interval >= 0,
         "sampled_update_interval must be zero or a positive integer"),
        (not (c.update_interval and c.sampled_update_interval),
         "exact and sampled route updates are mutually exclusive"),
        (0 < c.route_samples <= c.block_size, "route_samples must be in [1, block_size]"),
        (c.route_persistence >= 0, "route_persistence must be non-negative"),
        (c.bootstrap_mode in ("exact", "sampled"), "bootstrap_mode must be 'exact' or 'sampled'"),
        (c.dense_route_threshold is None or 0 < c.dense_route_threshold <= 1,
         "dense_route_threshold must be in (0, 1]"),
        (0 < c.keep <= 1, "keep must be in (0, 1]"),
        (0 < c.mass_target <= 1, "mass_target must be in (0, 1]"),
        (c.spatial_microtile_tokens > 0, "spatial_microtile_tokens must be positive"),
        (c.direction_min_ratio >= 0, "direction_min_ratio must be non-negative"),
        (c.direction_candidate_bonus >= 0, "direction_candidate_bonus must be non-negative"),
        (c.route_budget_scale > 0, "route_budget_scale must be positive"),
        (0 <= c.route_exploration_fraction <= 1, "route_exploration_fraction must be in [0, 1]"),
        (not c.directional_update or c.spatial_reorder,
         "directional_update requires spatial_reorder"),
    )
    for ok, message in checks:
        if not ok:
            raise ValueError(message)


class FlexReuseBackend:
    """Dense bootstrap followed by reuse with optional exact or sampled refresh.

    Each call is classified by ``_plan`` into one action (bootstrap, dense
    dispatch, exact refresh, inline sampled update, sparse reuse) that
    ``__call__`` runs; route bookkeeping lives in ``RouteState`` and the
    phase tally in ``PhaseLog``.  The decisions follow the reference's order
    (``flex.py:652-850``) so routes are refreshed at the same steps.
    """

    name = "flex_reuse"

    def __init__(self, config=None, routing_context=None, process_group=None):
        self.config = config or FlexReuseConfig()
        _validate(self.config)
        self._routing_context = routing_context
        self.process_group = process_group
        self.dense = DenseBackend()
        self.state = _StateTable()
        self.route_streams = {}
        self.spatial_layouts = {}
        self.pipelines = {}
        # head_parallel on CUDA: the chunks' packed inputs are pulled from the
        # ranks' shards and the attention stores into the ranks' output shards
        # over peer memory, instead of NCCL all-to-alls
        self.peer_exchange = True
        self.log = PhaseLog()

    @property
    def phase_counts(self):
        return self.log.counts

    @property
    def finished_routes(self):
        return [r._asdict() for r in self.log.released]

    def profile_summary(self):
        return self.log.summary(self.state.values())

    # ------------------------------------------------------------------ context
    def _context(self):
        if self._routing_context is not None:
            return self._routing_context(include_grid=True)
        # Resolved at call time so tests can monkeypatch this module's name.
        return globals()["routing_context"](include_grid=True)

    def _final_step(self, step):
        c = self.config
        return c.release_after_final_step and c.total_steps is not None and step >= c.total_steps - 1

    def _before_last_step(self, step):
        total = self.config.total_steps
        return total is None or step < total - 1

    # ------------------------------------------------------------------ dispatch
    def _global_keep(self, kept, numel):
        """Kept-block fraction over all heads of a layer/branch (all ranks)."""
        total = kept.sum()
        if self.process_group is not None:
            import torch.distributed as dist
            total = total.clone()
            dist.all_reduce(total, group=self.process_group)
            numel = numel * dist.get_world_size(self.process_group)
        return _fp32_mean_of_count(int(total.item()), numel)

    def _refresh_dispatch(self, state: RouteState):
        """Recompute the route's keep (and frontier) fraction; at or above
        ``dense_route_threshold`` the state goes dense for good and drops its
        route (``flex.py:473-493``)."""
        if state.route is None:
            state.keep = None
        else:
            kept = state.kept
            if kept is None:
                kept = state.route.reshape(state.route.shape[0], -1).sum(-1)
            state.keep = self._global_keep(kept, state.route.numel())
        f = state.frontier
        state.frontier_fraction = (None if f is None
                                   else _fp32_mean_of_count(int(f.sum().item()), f.numel()))
        threshold = self.config.dense_route_threshold
        state.dense = bool(threshold is not None and state.keep is not None
                           and state.keep >= threshold)
        if state.dense:
            state.drop_route()

    def _adopt_pending(self, state: RouteState):
        pending, state.pending = state.pending, None
        if pending is None:
            return
        torch.cuda.current_stream(pending.result.route.device).wait_event(pending.ready)
        state.adopt(pending.result, pending.source_step)
        self._refresh_dispatch(state)

    def _install(self, state: RouteState, result, tokens, step=None):
        if not isinstance(result, RouteResult):
            result = self._as_result(result, tokens)
        state.adopt(result, step)
        self._refresh_dispatch(state)

    def _as_result(self, mapping, tokens):
        """A RouteResult from a reference-style ``{"route": .., "frontier": ..}``
        mapping (a route producer substituted by a caller)."""
        route = mapping["route"]
        block_mask = mapping.get("block_mask")
        if block_mask is None:
            block_mask = _build_block_mask(route, tokens, self.config.block_size)
        return RouteResult(route, mapping.get("frontier"), mapping.get("kept"), block_mask)

    def _release(self, key):
        state = self.state.pop(key, None)
        if state is not None:
            self.log.release(state)

    # ------------------------------------------------------------------ routes
    def _sink_blocks(self, state):
        grid = state.get("grid")
        if not self.config.first_frame_sink or grid is None:
            return 0
        return math.ceil((grid[1] * grid[2]) / self.config.block_size)

    def _csr_result(self, result, tokens, layout):
        route = result.route.bool()
        frontier = None
        if layout is not None:
            frontier = frontier_mask(route, layout.neighbors(route.device))
        block_mask = BlockRoute(result.counts.unsqueeze(0), result.indices.unsqueeze(0), tokens,
                                self.config.block_size)
        return RouteResult(route, frontier, result.kept, block_mask)

    def _result_from_csr(self, state, result, tokens):
        return self._csr_result(result, tokens, state.get("layout"))

    def _sampled_route(self, state, q, k, softmax_scale):
        """Sampled mass, then either the directional frontier update or the
        prior + top-mass selection, with the sink and the CSR in the same
        kernel (``flex.py:508-548``)."""
        c = self.config
        mass = _sampled_block_mass(q, k, c.block_size, samples=c.route_samples,
                                   scale=softmax_scale, query_block_chunk=c.sample_query_block_chunk)
        previous, layout = state.get("route"), state.get("layout")
        tokens = q.shape[1]
        if c.directional_update and previous is not None and layout is not None:
            r = kernels.directional_update(
                mass, previous, layout.neighbors(mass.device), keep=c.keep,
                persistence=c.route_persistence, min_ratio=c.direction_min_ratio,
                candidate_bonus=c.direction_candidate_bonus, budget_scale=c.route_budget_scale,
                exploration_fraction=c.route_exploration_fraction,
                expand_q=c.direction_expand_q, expand_k=c.direction_expand_k,
                expand_joint=c.direction_expand_joint,
                previous_frontier=state.get("frontier"), sink_blocks=self._sink_blocks(state))
            csr = BlockRoute(r.counts.unsqueeze(0), r.indices.unsqueeze(0), tokens, c.block_size)
            return RouteResult(r.route, r.frontier, r.kept, csr)
        selected = kernels.route_select(
            mass, prev=previous if c.route_persistence else None, persistence=c.route_persistence,
            target=c.mass_target, keep=c.keep, sink_blocks=self._sink_blocks(state))
        return self._csr_result(selected, tokens, layout)

    def _exact_route(self, state, q, k, softmax_scale, mass=None):
        c = self.config
        if mass is None:
            mass = _block_attention_mass(q, k, None, c.block_size, scale=softmax_scale)
        selected = kernels.route_select(mass, target=c.mass_target, keep=c.keep,
                                        sink_blocks=self._sink_blocks(state))
        return self._csr_result(selected, q.shape[1], state.get("layout"))

    def _add_first_frame_sink(self, state, result):
        """Force the first latent frame's key blocks on in every row
        (``flex.py:550-566``); the selection kernels do this themselves, this
        helper serves routes built elsewhere."""
        sink = self._sink_blocks(state)
        if sink == 0:
            return result
        route = result["route"].clone()
        route[..., :sink] = True
        layout = state.get("layout")
        frontier = (frontier_mask(route, layout.neighbors(route.device)) if layout is not None
                    else result.get("frontier"))
        return {**dict(result), "route": route, "frontier": frontier, "kept": None,
                "block_mask": None}

    def _dense_with_mass(self, q, k, v, softmax_scale, dense_only):
        """Dense output plus its exact block mass from one attention pass; SDPA
        and no mass (computed later from q, k) for inputs that kernel does
        not take."""
        output, mass = _dense_and_mass(q, k, v, self.config.block_size, softmax_scale)
        if output is None:
            return self.dense(q, k, v, **dense_only), None
        return output, mass[0]

    def _spatial_layout(self, grid, tokens):
        c = self.config
        if not c.spatial_reorder or grid is None or math.prod(grid) != tokens:
            return None
        key = (tuple(grid), c.block_size, c.spatial_microtile_tokens)
        layout = self.spatial_layouts.get(key)
        if layout is None:
            layout = build_spatial_layout(grid, c.block_size, c.spatial_microtile_tokens)
            self.spatial_layouts[key] = layout
        return layout

    def _launch_side_route(self, state, q, k, step, softmax_scale):
        """Start the sampled route on the device's route stream after the work
        already queued on the current stream; adopted by the next call."""
        device = q.device
        side = self.route_streams.get(device)
        if side is None:
            side = self.route_streams[device] = torch.cuda.Stream(device=device)
        queued = torch.cuda.Event()
        queued.record(torch.cuda.current_stream(device))
        side.wait_event(queued)
        with torch.cuda.stream(side):
            q.record_stream(side)
            k.record_stream(side)
            result = self._sampled_route(state, q, k, softmax_scale)
            if not isinstance(result, RouteResult):
                result = self._as_result(result, q.shape[1])
            ready = torch.cuda.Event()
            ready.record(side)
        state.pending = PendingRoute(result, step, ready)

    def install_route(self, route, *, attention_id, branch, tokens, heads, head_dim, device,
                      grid=None, step=0):
        """Seed the reusable route of one layer and CFG branch.

        ``route``: bool ``[H, Qb, Kb]`` over route blocks in the backend's
        token order (Morton-packed when ``spatial_reorder`` is on).  The next
        call with this layer/branch at a later step reuses it exactly as a
        route produced by a bootstrap would be reused.  Returns the state.
        """
        layout = self._spatial_layout(grid, tokens)
        if self.config.spatial_reorder and layout is None:
            raise ValueError("spatial_reorder needs a grid whose product is the token count")
        route = route.to(device=device, dtype=torch.bool)
        key = (attention_id, branch, tokens, heads, head_dim, route.device,
               layout.signature if layout is not None else None)
        state = RouteState(step=step, layout=layout, grid=grid)
        frontier = (frontier_mask(route, layout.neighbors(route.device))
                    if layout is not None else None)
        self._install(state, RouteResult(route, frontier,
                                         route.reshape(route.shape[0], -1).sum(-1),
                                         _build_block_mask(route, tokens,
                                                           self.config.block_size)), tokens)
        self.state[key] = state
        return self.state[key]

    # ------------------------------------------------------------------ call
    def _dense_call(self, q, k, v, **kw):
        return self.dense(q, k, v, **kw)

    def packed_layout_for(self, tokens):
        """The spatial layout this backend's next call (under the current
        routing context) would pack its inputs with, or None.  A caller that
        already produced q, k, v in that order (the fused prologue) passes it
        back as ``packed_layout=`` and the backend skips its own reorder; the
        output is still returned in the original token order."""
        attention_id, _step, _branch, grid = self._context()
        if self.config.first_layer_dense and attention_id == 0:
            return None
        return self._spatial_layout(grid, tokens)

    def _plan(self, key, step):
        """The action for this call: "bootstrap", "dense", "exact_refresh",
        "sampled_update" (inline) or "reuse" / "reuse+prefetch"."""
        c = self.config
        state = self.state.get(key)
        if step == 0 or state is None:
            return "bootstrap"
        self._adopt_pending(state)
        if state.dense:
            return "dense"
        age = step - state.step
        if c.update_interval > 0 and age >= c.update_interval and not self._final_step(step):
            return "exact_refresh"
        if (c.sampled_update_interval > 0 and age >= c.sampled_update_interval
                and self._before_last_step(step)):
            return "reuse+prefetch" if c.prefetch_sampled_update else "sampled_update"
        return "reuse"

    def __call__(self, q, k, v, q_lens=None, k_lens=None, dropout_p=0.0, softmax_scale=None,
                 q_scale=None, causal=False, window_size=(-1, -1), deterministic=False,
                 dtype=torch.bfloat16, version=None, **kwargs):
        # Inputs already in route-block order of this layout (the fused
        # prologue's output, see packed_layout_for); not part of the
        # reference's signature, which swallows unknown keywords.
        packed = kwargs.pop("packed_layout", None)
        caller_kw = dict(q_lens=q_lens, k_lens=k_lens, dropout_p=dropout_p,
                         softmax_scale=softmax_scale, q_scale=q_scale, causal=causal,
                         window_size=window_size, deterministic=deterministic, dtype=dtype,
                         version=version, **kwargs)

        def as_called():
            # dense attention commutes with a token permutation: restore a
            # packed result to the caller's order
            out = self._dense_call(q, k, v, **caller_kw)
            return packed.restore(out.contiguous()) if packed is not None else out

        self_attention = q.shape[0] == 1 and q.shape[1] == k.shape[1]
        if not (self_attention and dropout_p == 0 and not causal and window_size == (-1, -1)):
            return as_called()
        attention_id, step, branch, grid = self._context()
        if self.config.first_layer_dense and attention_id == 0:
            self.log.hit("first_layer_dense")
            return as_called()
        layout = self._spatial_layout(grid, q.shape[1])
        if self.config.spatial_reorder and layout is None:
            return as_called()
        if packed is not None and (layout is None or packed.signature != layout.signature):
            q, k, v = (packed.restore(x.contiguous()) for x in (q, k, v))
            packed = None

        output_dtype = q.dtype
        q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
        if q_scale is not None:
            q = q * q_scale
        if layout is not None and packed is None:
            q, k, v = layout.reorder_qkv(q, k, v)
        key = (attention_id, branch, q.shape[1], q.shape[2], q.shape[3], q.device,
               layout.signature if layout is not None else None)
        dense_kw = dict(dropout_p=0.0, softmax_scale=softmax_scale, q_scale=None, causal=False,
                        window_size=(-1, -1), dtype=dtype)

        def unpacked(output):
            if layout is not None:
                output = layout.restore(output)
            return output.to(output_dtype)

        action = self._plan(key, step)
        if action == "bootstrap":
            output = self._bootstrap(key, step, layout, grid, q, k, v, softmax_scale, dense_kw)
        elif action == "dense":
            self.log.hit("dense_dispatch")
            output = self.dense(q, k, v, **dense_kw)
        elif action == "exact_refresh":
            state = self.state[key]
            output, mass = self._dense_with_mass(q, k, v, softmax_scale, dense_kw)
            self._install(state, self._exact_route(state, q, k, softmax_scale, mass), q.shape[1],
                          step)
            self.log.hit("exact_refresh")
        else:
            state = self.state[key]
            output = None
            if action == "sampled_update":
                state.block_mask = None
                self._install(state, self._sampled_route(state, q, k, softmax_scale), q.shape[1],
                              step)
                self.log.hit("sampled_update")
                if state.dense:
                    self.log.hit("dense_dispatch")
                    output = self.dense(q, k, v, **dense_kw)
            if output is None:
                # the output store writes raster order (the unpack is folded in)
                raster = _flex_output(q, k, v, state.block_mask, self.config.block_size,
                                      self.config.compile_kernel, scale=softmax_scale,
                                      out_rows=(layout.permutation(q.device)
                                                if layout is not None else None))
                self.log.hit("sparse_reuse")
                if action == "reuse+prefetch":
                    state.block_mask = None
                    self._launch_side_route(state, q, k, step, softmax_scale)
                    self.log.hit("sampled_update")
                if self._final_step(step):
                    self._release(key)
                return raster.to(output_dtype)
        if self._final_step(step):
            self._release(key)
        return unpacked(output)

    # ------------------------------------------------------------ multi-GPU
    def head_parallel(self, q, k, v, group, group_size, rows=None, chunks=None, **call_kw):
        """This backend over the head shards of sequence-sharded inputs.

        ``q, k, v``: ``[1, T/P, H, D]`` (one CFG branch of a sequence-parallel
        caller, ``P = group_size`` ranks in ``group``); returns the output
        shard ``[1, T/P, H, D]``.  A sparse-reuse call -- the common one --
        exchanges the heads in chunks overlapped with the attention
        (``parallel.PipelinedHeadParallel``): chunk c's heads attend over
        their slice of the layer's CSR route, packed by the exchange's row
        gather, and the kernel stores each output row into the output shard
        of the rank that holds its token (peer memory; ``peer_exchange``
        False: into the send buffer of an output all-to-all).  Every other call (bootstrap, refreshes, updates, dense
        dispatch, non-default arguments) exchanges all heads at once
        (``parallel.head_parallel_attention``) and runs ``__call__``.
        ``call_kw`` are ``__call__``'s keyword arguments.
        """
        from . import parallel

        if group_size == 1:
            return self(q, k, v, **call_kw)
        plan = self._reuse_plan(q, k, v, group_size, call_kw)
        if plan is None:
            return parallel.head_parallel_attention(
                q, k, v, lambda a, b, c: self(a, b, c, **call_kw), group, group_size, rows=rows)
        key, step, layout, state = plan
        heads = q.shape[2]
        pkey = (id(group), group_size, heads, q.shape[1], q.device,
                layout.signature if layout is not None else None, chunks)
        pipe = self.pipelines.get(pkey)
        if pipe is None:
            perm = layout.permutation_cpu if layout is not None else None
            inverse = layout.inverse_cpu if layout is not None else None
            pipe = parallel.PipelinedHeadParallel(group, group_size, heads, q.shape[1], perm,
                                                  inverse, chunks=chunks, rows=rows,
                                                  peer_out=self.peer_exchange and q.is_cuda,
                                                  peer_in=self.peer_exchange and q.is_cuda)
            self.pipelines[pkey] = pipe
        counts, indices = state.block_mask.counts[0], state.block_mask.indices[0]
        scale = call_kw.get("softmax_scale")

        def attend(qp, kp, vp, chunk, out, out_rows, peers=None):
            hs = pipe.chunk_slices()[chunk]     # the plan of the exchange in effect
            if peers is not None:
                kernels.block_sparse_attention_peers(qp, kp, vp, counts[hs], indices[hs], peers,
                                                     block=self.config.block_size, scale=scale,
                                                     out_rows=out_rows)
                return
            kernels.block_sparse_attention(qp, kp, vp, counts[hs], indices[hs],
                                           block=self.config.block_size, scale=scale, out=out,
                                           out_rows=out_rows)

        out = pipe(q, k, v, attend)
        self.log.hit("sparse_reuse")
        if self._final_step(step):
            self._release(key)
        return out

    def _reuse_plan(self, q, k, v, group_size, call_kw):
        """(key, step, layout, state) when the head-sharded call of these
        sequence shards is a plain sparse reuse, else None."""
        if set(call_kw) - {"softmax_scale", "dtype"}:
            return None
        if call_kw.get("dtype", torch.bfloat16) != q.dtype or q.dtype != torch.bfloat16:
            return None
        if not (q.shape == k.shape == v.shape and q.shape[0] == 1):
            return None
        b, t_local, h, d = q.shape
        if h % group_size:
            return None
        attention_id, step, branch, grid = self._context()
        if self.config.first_layer_dense and attention_id == 0:
            return None
        tokens = t_local * group_size
        layout = self._spatial_layout(grid, tokens)
        if self.config.spatial_reorder and layout is None:
            return None
        key = (attention_id, branch, tokens, h // group_size, d, q.device,
               layout.signature if layout is not None else None)
        if self._plan(key, step) != "reuse":
            return None
        state = self.state[key]
        if not isinstance(state.block_mask, BlockRoute):
            return None
        return key, step, layout, state

    def _bootstrap(self, key, step, layout, grid, q, k, v, softmax_scale, dense_kw):
        """Step 0 (or a new key): dense output plus the first route, exact
        from the same attention pass or sampled (``flex.py:706-762``)."""
        state = RouteState(step=step, layout=layout, grid=grid)
        self.state[key] = state
        if self.config.bootstrap_mode == "exact":
            output, mass = self._dense_with_mass(q, k, v, softmax_scale, dense_kw)
            self._install(state, self._exact_route(state, q, k, softmax_scale, mass), q.shape[1])
            self.log.hit("dense_bootstrap")
            return output
        output = self.dense(q, k, v, **dense_kw)
        if self.config.prefetch_sampled_bootstrap and self._before_last_step(step):
            self._launch_side_route(state, q, k, step, softmax_scale)
        else:
            self._install(state, self._sampled_route(state, q, k, softmax_scale), q.shape[1])
        self.log.hit("sampled_bootstrap")
        return output


def install_flex_reuse(config=None):
    """Return a configured backend (the reference's installer also patches Wan)."""
    return FlexReuseBackend(config)
