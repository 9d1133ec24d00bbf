"""Route decision restated in numpy (test oracle; see ``oracle/__init__``).

Each function cites the reference lines (yangshuo1230/DiT_Sparse_Atten,
``attention_backends/``) whose arithmetic it restates.  Floating-point steps
whose last bit decides the route follow the reference's PyTorch CPU evaluation
order exactly (``oracle.torch_cpu_order``).
"""

from __future__ import annotations

import math

import numpy as np

from . import torch_cpu_order as order


# ----------------------------------------------------------------------------
# bf16 helpers
# ----------------------------------------------------------------------------

def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest, ties to even), return float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint32).view(np.float32)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


# ----------------------------------------------------------------------------
# (a2) sampled block mass -- flex.py:205-251
# ----------------------------------------------------------------------------

def block_sizes(tokens: int, block: int) -> np.ndarray:
    """Valid tokens per route block (``flex.py:222-224``)."""
    blocks = math.ceil(tokens / block)
    ids = np.arange(blocks, dtype=np.int64)
    return np.minimum(tokens - ids * block, block)


def sample_indices(tokens: int, block: int, samples: int) -> np.ndarray:
    """Evenly spaced sample token ids ``[blocks, samples]`` (``flex.py:225-231``)."""
    if samples <= 0 or samples > block:
        raise ValueError("route_samples must be in [1, block_size]")
    sizes = block_sizes(tokens, block)
    s = np.arange(samples, dtype=np.int64)
    local = ((2 * s + 1)[None] * sizes[:, None]) // (2 * samples)
    local = np.minimum(local, sizes[:, None] - 1)
    return np.arange(len(sizes))[:, None] * block + local


def key_log_weights(tokens: int, block: int, samples: int) -> np.ndarray:
    """``log(size / samples)`` per sampled key, float32 (``flex.py:236-237``)."""
    sizes = block_sizes(tokens, block).astype(np.float32)
    w = np.log((sizes / np.float32(samples)).astype(np.float32)).astype(np.float32)
    return np.repeat(w, samples)


def sampled_block_mass(q, k, block, samples=2, scale=None, round_scores_bf16=True,
                       heads=None):
    """Sampled block mass for one batch element (``flex.py:205-251``).

    ``q``/``k``: float32 arrays ``[T, H, D]`` holding the (bf16) inputs.
    ``round_scores_bf16`` reproduces the bf16 matmul output and the bf16
    ``* score_scale`` of the reference (``flex.py:245``).  Returns float32
    ``[H, Qb, Kb]``.  ``heads`` optionally restricts the computation.
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    tokens, nheads, dim = q.shape
    idx = sample_indices(tokens, block, samples)
    blocks = idx.shape[0]
    flat = idx.reshape(-1)
    lw = key_log_weights(tokens, block, samples)
    s = np.float32(scale if scale is not None else dim ** -0.5)
    heads = range(nheads) if heads is None else heads
    out = []
    for h in heads:
        sq = q[flat, h]                      # [Qb*S, D]
        sk = k[flat, h]
        acc = sq @ sk.T                      # fp32 accumulate
        if round_scores_bf16:
            scores = round_bf16(round_bf16(acc) * s)
        else:
            scores = (acc * s).astype(np.float32)
        x = (scores + lw[None]).astype(np.float32)
        x = x - x.max(-1, keepdims=True)
        e = np.exp(x, dtype=np.float32)
        p = (e / e.sum(-1, keepdims=True, dtype=np.float32)).astype(np.float32)
        m = p.reshape(blocks, samples, blocks, samples).sum(-1, dtype=np.float32)
        out.append((m.sum(1, dtype=np.float32) / np.float32(samples)).astype(np.float32))
    return np.stack(out)


def exact_block_mass(q, k, lse, block, scale=None):
    """Exact dense block mass from Q, K and per-query LSE (``flex.py:97-108``).

    ``q``/``k``: ``[T, H, D]``; ``lse``: ``[H, T]``.  Returns ``[H, Qb, Kb]``.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    tokens, heads, dim = q.shape
    s = scale if scale is not None else dim ** -0.5
    blocks = math.ceil(tokens / block)
    pad = blocks * block - tokens
    out = np.zeros((heads, blocks, blocks))
    for h in range(heads):
        p = np.exp(q[:, h] @ k[:, h].T * s - np.asarray(lse, np.float64)[h][:, None])
        p = np.pad(p, ((0, pad), (0, pad)))
        out[h] = p.reshape(blocks, block, blocks, block).sum((1, 3))
    return out.astype(np.float32)


# ----------------------------------------------------------------------------
# (a3) persistence prior -- flex.py:535-541
# ----------------------------------------------------------------------------

def persistence_prior(mass, previous, persistence):
    """``mass + persistence * mass.mean(-1, keepdim=True) * previous.float()``."""
    mass = np.asarray(mass, np.float32)
    if not persistence or previous is None:
        return mass
    bump = order.mul_scalar(order.row_mean(mass), persistence)[..., None]
    prev = np.asarray(previous, bool)
    return np.where(prev, (mass + bump).astype(np.float32),
                    (mass + np.float32(0)).astype(np.float32)).astype(np.float32)


# ----------------------------------------------------------------------------
# (a4) top-mass selection -- flex.py:83-94 (same rule sparse.py:171-181)
# ----------------------------------------------------------------------------

def selection_order(mass: np.ndarray) -> np.ndarray:
    """``mass.argsort(-1, descending=True)`` exactly as the reference's CPU build.

    The sort is unstable: equal values are ordered the way libstdc++'s
    introsort leaves them (``oracle/csrc/torch_cpu_sort.c``).  Only rows where
    equal values straddle the selection cut (``boundary_ties``) depend on it.
    """
    import ctypes

    from .build import load

    mass = np.ascontiguousarray(mass, dtype=np.float32)
    n = mass.shape[-1]
    rows = mass.size // n if n else 0
    order = np.empty(mass.shape, np.int32)
    scratch = np.empty(max(1, n) * 2, np.int32)
    if rows:
        load().oracle_argsort_desc(mass.ctypes.data_as(ctypes.c_void_p), rows, n,
                                   order.ctypes.data_as(ctypes.c_void_p),
                                   scratch.ctypes.data_as(ctypes.c_void_p))
    return order.astype(np.int64)


def top_mass_counts(mass, target, keep):
    """Per-row kept count before the cap is applied, and the cap."""
    mass = np.asarray(mass, np.float32)
    cols = mass.shape[-1]
    srt = np.take_along_axis(mass, selection_order(mass), -1)
    threshold = order.mul_scalar(order.row_sum(mass), target)[..., None]
    counts = (order.cumsum(srt) < threshold).sum(-1) + 1
    cap = max(1, math.ceil(cols * keep))
    return counts, cap


def top_mass_route(mass, target, keep):
    """Boolean route ``[..., Kb]`` from ``_top_mass_route`` (``flex.py:83-94``)."""
    mass = np.asarray(mass, np.float32)
    counts, cap = top_mass_counts(mass, target, keep)
    counts = np.minimum(counts, cap)
    idx = selection_order(mass)
    ranks = np.empty_like(idx)
    np.put_along_axis(ranks, idx, np.broadcast_to(np.arange(mass.shape[-1]), idx.shape), -1)
    return ranks < counts[..., None]


def boundary_ties(mass, target, keep):
    """Rows whose kept set depends on the tie order (tied values straddle the cut)."""
    mass = np.asarray(mass, np.float32)
    counts, cap = top_mass_counts(mass, target, keep)
    counts = np.minimum(counts, cap)
    srt = np.take_along_axis(mass, selection_order(mass), -1)
    n = mass.shape[-1]
    c = counts[..., None]
    last_in = np.take_along_axis(srt, np.clip(c - 1, 0, n - 1), -1)
    first_out = np.take_along_axis(srt, np.clip(c, 0, n - 1), -1)
    return ((c < n) & (last_in == first_out))[..., 0]


# ----------------------------------------------------------------------------
# (a5) first-frame key sink -- flex.py:550-566
# ----------------------------------------------------------------------------

def first_frame_blocks(grid, block):
    return math.ceil((grid[1] * grid[2]) / block)


def add_first_frame_sink(route, grid, block):
    route = np.array(route, bool, copy=True)
    route[..., : first_frame_blocks(grid, block)] = True
    return route


# ----------------------------------------------------------------------------
# (a6) dense-dispatch keep -- flex.py:473-493
# ----------------------------------------------------------------------------

def route_keep(route) -> float:
    """``float(route.float().mean())``: float32 ``count / numel``."""
    route = np.asarray(route, bool)
    return float(np.float32(np.float32(route.sum()) / np.float32(route.size)))


# ----------------------------------------------------------------------------
# (a7) CSR pack -- flex.py:275-281, layout_ops.py:128-151
# ----------------------------------------------------------------------------

def pack_boolean_rows(route):
    """Counts and ids: selected ids ascending, then unselected ids ascending."""
    route = np.asarray(route, bool)
    counts = route.sum(-1).astype(np.int32)
    indices = np.argsort(~route, axis=-1, kind="stable").astype(np.int32)
    return counts, indices


# ----------------------------------------------------------------------------
# composite: flex.py:508-566 (non-directional sampled route)
# ----------------------------------------------------------------------------

def sampled_route(mass, previous, persistence, target, keep, grid=None, block=128,
                  first_frame_sink=True):
    prior = persistence_prior(mass, previous, persistence)
    route = top_mass_route(prior, target, keep)
    if first_frame_sink and grid is not None:
        route = add_first_frame_sink(route, grid, block)
    return route


# ----------------------------------------------------------------------------
# (f3) directional frontier update -- routing.py:10-168
# Arrays are [..., Q, K] with Q == K (one plane per head); neighbours [K, 4]
# int, -1 where a block has no spatial neighbour in that direction.
# ----------------------------------------------------------------------------

def frontier_mask(route, neighbors):
    """Selected cells with an unselected valid neighbour along Q or K
    (``routing.py:10-43``)."""
    route = np.asarray(route, bool)
    nb = np.asarray(neighbors, np.int64)
    valid = nb >= 0
    safe = np.maximum(nb, 0)
    q_sel = route[..., safe, :]                                # [..., Q, 4, K]
    open_q = (valid[:, :, None] & ~q_sel).any(-2)
    k_sel = route[..., :, safe]                                # [..., Q, K, 4]
    open_k = (valid & ~k_sel).any(-1)
    return route & (open_q | open_k)


def _best_targets(mass, route, neighbors, frontier, axis, min_ratio):
    """Per frontier cell, the best unselected neighbour along ``axis`` (1 = Q,
    2 = K) and whether it is eligible (``routing.py:55-84``).  The first of
    equal maxima wins, as ``Tensor.max(-1)``."""
    nb = np.asarray(neighbors, np.int64)
    valid = nb >= 0
    safe = np.maximum(nb, 0)
    if axis == 1:
        values = np.moveaxis(mass[..., safe, :], -2, -1)       # [..., Q, K, 4]
        sel = np.moveaxis(route[..., safe, :], -2, -1)
        ok = valid[:, None, :]
        targets = np.broadcast_to(safe[:, None, :], values.shape)
    else:
        values = mass[..., :, safe]
        sel = route[..., :, safe]
        ok = valid[None, :, :]
        targets = np.broadcast_to(safe[None, :, :], values.shape)
    values = np.where(ok & ~sel, values, np.float32(-np.inf)).astype(np.float32)
    direction = values.argmax(-1)
    best = np.take_along_axis(values, direction[..., None], -1)[..., 0]
    target = np.take_along_axis(targets, direction[..., None], -1)[..., 0]
    eligible = frontier & np.isfinite(best) & (best >= order.mul_scalar(mass, min_ratio))
    return target, eligible


def _rank_below(values, counts):
    """``ranks(values.argsort(-1, descending=True)) < counts`` with the
    reference's tie order (``routing.py:87-94``, ``:145-148``)."""
    idx = selection_order(values)
    ranks = np.empty_like(idx)
    np.put_along_axis(ranks, idx, np.broadcast_to(np.arange(values.shape[-1]), idx.shape), -1)
    return ranks < np.asarray(counts)[..., None]


def directional_budget_update(mass, previous, neighbors, *, keep, persistence=0.5,
                              min_ratio=0.0, candidate_bonus=0.0, budget_scale=1.0,
                              exploration_fraction=0.0, expand_q=True, expand_k=True,
                              expand_joint=True, previous_frontier=None):
    """``directional_budget_update`` (``routing.py:97-168``): expand the
    previous route's frontier by one best neighbour per cell along Q, K and
    both, optionally add the best-mass cells outside the pool, then keep a
    per-row budget of the highest prior scores inside the pool."""
    mass = np.asarray(mass, np.float32)
    prev = np.asarray(previous, bool)
    blocks = mass.shape[-1]
    front = (np.asarray(previous_frontier, bool) if previous_frontier is not None
             else frontier_mask(prev, neighbors))
    tq, eq = _best_targets(mass, prev, neighbors, front, 1, min_ratio)
    tk, ek = _best_targets(mass, prev, neighbors, front, 2, min_ratio)
    lead = np.indices(mass.shape)
    planes = tuple(lead[:-2])
    q_idx, k_idx = lead[-2], lead[-1]
    cand = np.zeros(mass.shape, bool)
    if expand_q:
        cand[tuple(p[eq] for p in planes) + (tq[eq], k_idx[eq])] = True
    if expand_k:
        cand[tuple(p[ek] for p in planes) + (q_idx[ek], tk[ek])] = True
    if expand_joint:
        j = eq & ek
        cand[tuple(p[j] for p in planes) + (tq[j], tk[j])] = True
    cand &= ~prev
    pool = prev | cand
    exploration = np.zeros_like(pool)
    if exploration_fraction:
        count = max(1, math.ceil(blocks * exploration_fraction))
        masked = np.where(pool, np.float32(-np.inf), mass).astype(np.float32)
        exploration = _rank_below(masked, np.full(mass.shape[:-1], count))
        pool = pool | exploration
    row_scale = order.row_mean(mass)[..., None]
    score = (mass + order.mul_scalar(row_scale, persistence) * prev.astype(np.float32)
             ).astype(np.float32)
    if candidate_bonus:
        score = (score + order.mul_scalar(row_scale, candidate_bonus)
                 * cand.astype(np.float32)).astype(np.float32)
    cap = max(1, math.ceil(blocks * keep))
    counts = np.ceil(prev.sum(-1).astype(np.float32) * np.float32(budget_scale))
    counts = np.clip(counts.astype(np.int64), 1, cap)
    counts = np.maximum(np.minimum(counts, pool.sum(-1)), 1)
    masked = np.where(pool, score, np.float32(-np.inf)).astype(np.float32)
    route = _rank_below(masked, counts) & pool
    return {
        "route": route,
        "frontier": frontier_mask(route, neighbors),
        "candidates": cand,
        "exploration": exploration,
        "dropped": prev & ~route,
        "added": route & ~prev,
    }


def directional_route(mass, previous, neighbors, grid=None, block=128, first_frame_sink=True,
                      **kw):
    """The directional branch of ``_sampled_route`` (``flex.py:517-534``)
    followed by ``_add_first_frame_sink`` (``flex.py:550-566``), which also
    recomputes the frontier of the sunk route."""
    result = directional_budget_update(mass, previous, neighbors, **kw)
    if first_frame_sink and grid is not None:
        result = dict(result)
        result["route"] = add_first_frame_sink(result["route"], grid, block)
        result["frontier"] = frontier_mask(result["route"], neighbors)
    return result
