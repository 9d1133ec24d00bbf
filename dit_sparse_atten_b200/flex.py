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
from dataclasses import dataclass

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


class FlexReuseBackend:
    """Dense bootstrap followed by reuse with optional exact or sampled refresh."""

    name = "flex_reuse"

    def __init__(self, config=None, routing_context=None, process_group=None):
        self.config = config or FlexReuseConfig()
        c = self.config
        if c.block_size != 128:
            raise ValueError("The minimal flex_reuse backend currently supports only 128-token blocks")
        if c.update_interval < 0:
            raise ValueError("update_interval must be zero or a positive integer")
        if c.sampled_update_interval < 0:
            raise ValueError("sampled_update_interval must be zero or a positive integer")
        if c.update_interval and c.sampled_update_interval:
            raise ValueError("exact and sampled route updates are mutually exclusive")
        if not 0 < c.route_samples <= c.block_size:
            raise ValueError("route_samples must be in [1, block_size]")
        if c.route_persistence < 0:
            raise ValueError("route_persistence must be non-negative")
        if c.bootstrap_mode not in ("exact", "sampled"):
            raise ValueError("bootstrap_mode must be 'exact' or 'sampled'")
        if c.dense_route_threshold is not None and not 0 < c.dense_route_threshold <= 1:
            raise ValueError("dense_route_threshold must be in (0, 1]")
        if not 0 < c.keep <= 1:
            raise ValueError("keep must be in (0, 1]")
        if not 0 < c.mass_target <= 1:
            raise ValueError("mass_target must be in (0, 1]")
        if c.spatial_microtile_tokens <= 0:
            raise ValueError("spatial_microtile_tokens must be positive")
        if c.direction_min_ratio < 0:
            raise ValueError("direction_min_ratio must be non-negative")
        if c.direction_candidate_bonus < 0:
            raise ValueError("direction_candidate_bonus must be non-negative")
        if c.route_budget_scale <= 0:
            raise ValueError("route_budget_scale must be positive")
        if not 0 <= c.route_exploration_fraction <= 1:
            raise ValueError("route_exploration_fraction must be in [0, 1]")
        if c.directional_update and not c.spatial_reorder:
            raise ValueError("directional_update requires spatial_reorder")
        self._routing_context = routing_context
        self.process_group = process_group
        self.dense = DenseBackend()
        self.state = {}
        self.route_streams = {}
        self.spatial_layouts = {}
        self.phase_counts = {
            "dense_bootstrap": 0,
            "sampled_bootstrap": 0,
            "exact_refresh": 0,
            "sampled_update": 0,
            "sparse_reuse": 0,
            "dense_dispatch": 0,
            "first_layer_dense": 0,
        }
        self.finished_routes = []

    # ------------------------------------------------------------------ context
    def _context(self):
        if self._routing_context is not None:
            return self._routing_context(include_grid=True)
        # Resolved at call time so tests can monkeypatch this module's name.
        return globals()["routing_context"](include_grid=True)

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

    def _activate_pending_route(self, state):
        pending = state.pop("pending", None)
        if pending is None:
            return
        torch.cuda.current_stream(pending["route"].device).wait_event(pending["ready"])
        state.update({
            "route": pending["route"],
            "frontier": pending.get("frontier"),
            "block_mask": pending["block_mask"],
            "kept": pending.get("kept"),
            "step": pending["source_step"],
        })
        self._update_dispatch(state)

    def _update_dispatch(self, state):
        threshold = self.config.dense_route_threshold
        route = state.get("route")
        keep = None
        if route is not None:
            kept = state.get("kept")
            if kept is None:
                kept = route.reshape(route.shape[0], -1).sum(-1)
            keep = self._global_keep(kept, route.numel())
        state["keep"] = keep
        frontier = state.get("frontier")
        state["frontier_fraction"] = (
            _fp32_mean_of_count(int(frontier.sum().item()), frontier.numel())
            if frontier is not None else None)
        state["dense"] = bool(threshold is not None and keep is not None and keep >= threshold)
        if state["dense"]:
            state["route"] = None
            state["block_mask"] = None
            state["frontier"] = None
            state["kept"] = None

    def _is_final_step(self, step):
        return (self.config.release_after_final_step and self.config.total_steps is not None
                and step >= self.config.total_steps - 1)

    def _release_route(self, key, state):
        self.finished_routes.append({
            "keep": state.get("keep"),
            "frontier_fraction": state.get("frontier_fraction"),
            "dense": bool(state.get("dense")),
        })
        self.state.pop(key, None)

    # ------------------------------------------------------------------ routes
    def _sink_blocks(self, state):
        grid = state.get("grid")
        if not self.config.first_frame_sink or grid is None:
            return 0
        return math.ceil((grid[1] * grid[2]) / self.config.block_size)

    def _sampled_route(self, state, q, k, softmax_scale):
        """Sampled mass -> prior -> top-mass -> sink -> CSR in two kernels."""
        c = self.config
        mass = _sampled_block_mass(q, k, c.block_size, samples=c.route_samples,
                                   scale=softmax_scale, query_block_chunk=c.sample_query_block_chunk)
        previous = state.get("route")
        layout = state.get("layout")
        if c.directional_update and previous is not None and layout is not None:
            # flex.py:517-534 + the sink of :550-566, in one call
            r = kernels.directional_update(
                mass, previous, layout.neighbors(mass.device), keep=c.keep,
                persistence=c.route_persistence, min_ratio=c.direction_min_ratio,
                candidate_bonus=c.direction_candidate_bonus, budget_scale=c.route_budget_scale,
                exploration_fraction=c.route_exploration_fraction,
                expand_q=c.direction_expand_q, expand_k=c.direction_expand_k,
                expand_joint=c.direction_expand_joint,
                previous_frontier=state.get("frontier"), sink_blocks=self._sink_blocks(state))
            return {
                "route": r.route,
                "frontier": r.frontier,
                "kept": r.kept,
                "block_mask": BlockRoute(r.counts.unsqueeze(0), r.indices.unsqueeze(0),
                                         q.shape[1], c.block_size),
            }
        result = kernels.route_select(
            mass, prev=previous if c.route_persistence else None,
            persistence=c.route_persistence, target=c.mass_target, keep=c.keep,
            sink_blocks=self._sink_blocks(state))
        return self._result_from_csr(state, result, q.shape[1])

    def _result_from_csr(self, state, result, tokens):
        route = result.route.bool()
        layout = state.get("layout")
        frontier = frontier_mask(route, layout.neighbors(route.device)) if layout is not None else None
        return {
            "route": route,
            "frontier": frontier,
            "kept": result.kept,
            "block_mask": BlockRoute(result.counts.unsqueeze(0), result.indices.unsqueeze(0),
                                     tokens, self.config.block_size),
        }

    def _add_first_frame_sink(self, state, result):
        if not self.config.first_frame_sink:
            return result
        grid = state.get("grid")
        if grid is None:
            return result
        route = result["route"].clone()
        route[..., :math.ceil((grid[1] * grid[2]) / self.config.block_size)] = True
        result = dict(result)
        result["route"] = route
        result.pop("kept", None)
        result.pop("block_mask", None)
        layout = state.get("layout")
        if layout is not None:
            result["frontier"] = frontier_mask(route, layout.neighbors(route.device))
        return result

    def _dense_for_exact_route(self, q, k, v, softmax_scale, dense_only):
        """Dense output plus its exact block mass from one attention pass, or
        SDPA and no mass (computed later from q, k) for inputs that kernel
        does not take."""
        output, mass = _dense_and_mass(q, k, v, self.config.block_size, softmax_scale)
        if output is None:
            return self.dense(q, k, v, **dense_only), None
        return output, mass[0]

    def _exact_route(self, state, q, k, softmax_scale, mass=None):
        c = self.config
        if mass is None:
            mass = _block_attention_mass(q, k, None, c.block_size, scale=softmax_scale)
        result = kernels.route_select(mass, target=c.mass_target, keep=c.keep,
                                      sink_blocks=self._sink_blocks(state))
        return self._result_from_csr(state, result, q.shape[1])

    def _install_route(self, state, result, tokens):
        block_mask = result.get("block_mask")
        if block_mask is None:
            block_mask = _build_block_mask(result["route"], tokens, self.config.block_size)
        state.update({
            "route": result["route"],
            "frontier": result.get("frontier"),
            "kept": result.get("kept"),
            "block_mask": block_mask,
        })

    def _spatial_layout(self, grid, tokens):
        if not self.config.spatial_reorder:
            return None
        if grid is None or math.prod(grid) != tokens:
            return None
        key = (tuple(grid), self.config.block_size, self.config.spatial_microtile_tokens)
        if key not in self.spatial_layouts:
            self.spatial_layouts[key] = build_spatial_layout(
                grid, self.config.block_size, self.config.spatial_microtile_tokens)
        return self.spatial_layouts[key]

    def _prefetch_sampled_route(self, state, q, k, step, softmax_scale, phase="sampled_update"):
        stream = self.route_streams.setdefault(q.device, torch.cuda.Stream(device=q.device))
        attention_done = torch.cuda.Event()
        attention_done.record(torch.cuda.current_stream(q.device))
        stream.wait_event(attention_done)
        with torch.cuda.stream(stream):
            q.record_stream(stream)
            k.record_stream(stream)
            result = self._sampled_route(state, q, k, softmax_scale)
            ready = torch.cuda.Event()
            ready.record(stream)
        state["pending"] = {
            "route": result["route"],
            "frontier": result.get("frontier"),
            "kept": result.get("kept"),
            "block_mask": result["block_mask"],
            "source_step": step,
            "ready": ready,
        }
        self.phase_counts[phase] += 1

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
        state = {"route": route, "frontier": None, "step": step, "layout": layout, "grid": grid,
                 "kept": route.reshape(route.shape[0], -1).sum(-1),
                 "block_mask": _build_block_mask(route, tokens, self.config.block_size)}
        if layout is not None:
            state["frontier"] = frontier_mask(route, layout.neighbors(route.device))
        self._update_dispatch(state)
        self.state[key] = state
        return state

    def profile_summary(self):
        active = [s for s in self.state.values() if s.get("route") is not None]
        keep = [s.get("keep") for s in active] + [
            s["keep"] for s in self.finished_routes if s["keep"] is not None]
        frontier = [s.get("frontier_fraction") for s in active] + [
            s["frontier_fraction"] for s in self.finished_routes
            if s["frontier_fraction"] is not None]
        return {
            "phase_counts": dict(self.phase_counts),
            "active_routes": len(active),
            "released_routes": len(self.finished_routes),
            "mean_route_keep": sum(keep) / len(keep) if keep else None,
            "mean_frontier_fraction": sum(frontier) / len(frontier) if frontier else None,
            "dense_dispatched_routes": sum(bool(s.get("dense")) for s in self.state.values())
            + sum(s["dense"] for s in self.finished_routes),
        }

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

    def __call__(self, q, k, v, q_lens=None, k_lens=None, dropout_p=0.0, softmax_scale=None,
                 q_scale=None, causal=False, window_size=(-1, -1), deterministic=False,
                 dtype=torch.bfloat16, version=None, **kwargs):
        # Inputs already in route-block order of this layout (the fused
        # prologue's output, see packed_layout_for); not part of the
        # reference's signature, which swallows unknown keywords.
        packed = kwargs.pop("packed_layout", None)
        dense_kw = dict(q_lens=q_lens, k_lens=k_lens, dropout_p=dropout_p,
                        softmax_scale=softmax_scale, q_scale=q_scale, causal=causal,
                        window_size=window_size, deterministic=deterministic, dtype=dtype,
                        version=version, **kwargs)

        def dense_unpacked():
            # dense attention is order-equivariant: restore a packed result
            out = self._dense_call(q, k, v, **dense_kw)
            return packed.restore(out.contiguous()) if packed is not None else out

        supported = (q.shape[0] == 1 and q.shape[1] == k.shape[1] and dropout_p == 0
                     and not causal and window_size == (-1, -1))
        if not supported:
            return dense_unpacked()

        attention_id, step, branch, grid = self._context()
        if self.config.first_layer_dense and attention_id == 0:
            self.phase_counts["first_layer_dense"] += 1
            return dense_unpacked()
        layout = self._spatial_layout(grid, q.shape[1])
        if self.config.spatial_reorder and layout is None:
            return dense_unpacked()
        if packed is not None and (layout is None or packed.signature != layout.signature):
            q, k, v = (packed.restore(x.contiguous()) for x in (q, k, v))
            packed = None

        output_dtype = q.dtype
        q = q.to(dtype)
        k = k.to(dtype)
        v = v.to(dtype)
        if q_scale is not None:
            q = q * q_scale
        if layout is not None and packed is None:
            q, k, v = layout.reorder_qkv(q, k, v)

        def finish(output):
            if layout is not None:
                output = layout.restore(output)
            return output.to(output_dtype)

        key = (attention_id, branch, q.shape[1], q.shape[2], q.shape[3], q.device,
               layout.signature if layout is not None else None)
        dense_only = dict(dropout_p=0.0, softmax_scale=softmax_scale, q_scale=None,
                          causal=False, window_size=(-1, -1), dtype=dtype)
        if step == 0 or key not in self.state:
            state = {"route": None, "frontier": None, "block_mask": None, "step": step,
                     "layout": layout, "grid": grid}
            if self.config.bootstrap_mode == "exact":
                output, mass = self._dense_for_exact_route(q, k, v, softmax_scale, dense_only)
                self.state[key] = state
                self._install_route(state, self._exact_route(state, q, k, softmax_scale, mass),
                                    q.shape[1])
                self._update_dispatch(state)
                self.phase_counts["dense_bootstrap"] += 1
            else:
                output = self.dense(q, k, v, **dense_only)
                self.state[key] = state
                if (self.config.prefetch_sampled_bootstrap
                        and (self.config.total_steps is None
                             or step < self.config.total_steps - 1)):
                    self._prefetch_sampled_route(state, q, k, step, softmax_scale,
                                                 phase="sampled_bootstrap")
                else:
                    self._install_route(state, self._sampled_route(state, q, k, softmax_scale),
                                        q.shape[1])
                    self._update_dispatch(state)
                    self.phase_counts["sampled_bootstrap"] += 1
            if self._is_final_step(step):
                self._release_route(key, self.state[key])
            return finish(output)

        state = self.state[key]
        self._activate_pending_route(state)
        if state.get("dense"):
            self.phase_counts["dense_dispatch"] += 1
            output = self.dense(q, k, v, **dense_only).to(output_dtype)
            if self._is_final_step(step):
                self._release_route(key, state)
            return finish(output)
        if (self.config.update_interval > 0
                and (step - state["step"]) >= self.config.update_interval
                and not self._is_final_step(step)):
            output, mass = self._dense_for_exact_route(q, k, v, softmax_scale, dense_only)
            self._install_route(state, self._exact_route(state, q, k, softmax_scale, mass),
                                q.shape[1])
            state["step"] = step
            self._update_dispatch(state)
            self.phase_counts["exact_refresh"] += 1
            return finish(output)

        sampled_update_due = (
            self.config.sampled_update_interval > 0
            and (step - state["step"]) >= self.config.sampled_update_interval
            and (self.config.total_steps is None or step < self.config.total_steps - 1))
        if sampled_update_due and not self.config.prefetch_sampled_update:
            state["block_mask"] = None
            self._install_route(state, self._sampled_route(state, q, k, softmax_scale), q.shape[1])
            state["step"] = step
            self._update_dispatch(state)
            self.phase_counts["sampled_update"] += 1
            if state.get("dense"):
                self.phase_counts["dense_dispatch"] += 1
                return finish(self.dense(q, k, v, **dense_only))

        # The sparse output goes straight back to raster order (no unpack pass).
        output = _flex_output(q, k, v, state["block_mask"], self.config.block_size,
                              self.config.compile_kernel, scale=softmax_scale,
                              out_rows=layout.permutation(q.device) if layout is not None
                              else None)
        self.phase_counts["sparse_reuse"] += 1
        if self.config.prefetch_sampled_update and sampled_update_due:
            state["block_mask"] = None
            self._prefetch_sampled_route(state, q, k, step, softmax_scale)
        if self._is_final_step(step):
            self._release_route(key, state)
        return output.to(output_dtype)


def install_flex_reuse(config=None):
    """Return a configured backend (the reference's installer also patches Wan)."""
    return FlexReuseBackend(config)
