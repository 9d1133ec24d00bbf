"""Frontier-aware route updates on the GPU (``attention_backends/routing.py``
of the reference, same names, arguments and error messages).

``frontier_mask`` and ``directional_budget_update`` run as CUDA kernels
(``csrc/directional.cu``) through the C ABI; they take CUDA tensors and raise
on anything else.  The results are bit-identical to the reference's PyTorch
code from the same inputs, including which of several equal scores is kept.
"""

from __future__ import annotations

import torch

from . import kernels


def frontier_mask(route: torch.Tensor, neighbors: torch.Tensor) -> torch.Tensor:
    """Selected route cells adjacent to an unselected spatial cell
    (``routing.py:37-43``); ``route`` bool ``[H, Qb, Kb]``, ``neighbors``
    ``[Kb, 4]`` with -1 for a missing neighbour."""
    return kernels.frontier_mask(route, neighbors)


def directional_budget_update(mass, previous, neighbors, *, keep, persistence=0.5,
                              min_ratio=0.0, candidate_bonus=0.0, budget_scale=1.0,
                              exploration_fraction=0.0, expand_q=True, expand_k=True,
                              expand_joint=True, previous_frontier=None):
    """Expand only route frontiers, then prune back to a per-row budget
    (``routing.py:97-168``).  Returns the reference's dict: ``route``,
    ``frontier``, ``candidates``, ``exploration``, ``dropped``, ``added``."""
    if previous.shape != mass.shape:
        raise ValueError("previous route and mass must have identical shapes")
    if tuple(neighbors.shape) != (mass.shape[-1], 4):
        raise ValueError("neighbors must have shape [blocks, 4]")
    if budget_scale <= 0:
        raise ValueError("budget_scale must be positive")
    if not 0 <= exploration_fraction <= 1:
        raise ValueError("exploration_fraction must be in [0, 1]")
    r = kernels.directional_update(
        mass, previous, neighbors, keep=keep, persistence=persistence, min_ratio=min_ratio,
        candidate_bonus=candidate_bonus, budget_scale=budget_scale,
        exploration_fraction=exploration_fraction, expand_q=expand_q, expand_k=expand_k,
        expand_joint=expand_joint, previous_frontier=previous_frontier)
    return {"route": r.route, "frontier": r.frontier, "candidates": r.candidates,
            "exploration": r.exploration, "dropped": r.dropped, "added": r.added}
