"""Per-call routing context: attention layer id, denoising step, CFG branch, grid.

Mirrors ``attention_backends/context.py:24-49`` of the reference: a module-level
``_STATE`` that the model frontend writes before each self-attention call and
``routing_context()`` that the backend reads.  A frontend that already owns a
context (for example the reference's own ``attention_backends.context``) can be
handed to ``FlexReuseBackend(routing_context=...)`` instead.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class _RuntimeState:
    attention_id: int = -1
    denoising_step: int = -1
    cfg_branch: int = -1
    grid_size: tuple | None = None
    last_timestep: float | None = None
    forward_calls: list = field(default_factory=list)


_STATE = _RuntimeState()


def reset_runtime_state():
    """Reset per-generation routing state."""
    global _STATE
    _STATE = _RuntimeState()


def set_routing_context(attention_id=None, step=None, branch=None, grid=None):
    """Update the fields a frontend publishes before an attention call."""
    if attention_id is not None:
        _STATE.attention_id = int(attention_id)
    if step is not None:
        _STATE.denoising_step = int(step)
    if branch is not None:
        _STATE.cfg_branch = int(branch)
    if grid is not None:
        _STATE.grid_size = tuple(int(v) for v in grid)


def routing_context(include_grid=False):
    values = (_STATE.attention_id, _STATE.denoising_step, _STATE.cfg_branch)
    return values + (_STATE.grid_size,) if include_grid else values
