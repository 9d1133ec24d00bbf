"""B200-native routed block-sparse self-attention for Wan video DiTs.

A drop-in for the ``flex_reuse`` attention backend of the reference study
(yangshuo1230/DiT_Sparse_Atten): the same backend callable and configuration,
with the block-sparse attention, the sampled/exact route decision and the
Morton spatial reorder running as hand-written sm_100a kernels in
``libbsa.so`` (C ABI: ``include/bsa.h``).

Public surface:
  FlexReuseBackend, FlexReuseConfig     the backend (``flex.py``)
  DenseBackend                          SDPA fallback (``dense.py``)
  routing_context, set_routing_context  per-call context (``context.py``)
  build_spatial_layout                  Morton layout (``spatial.py``)
  get_backend(name, **config)           registry: "dense", "flex_reuse"
  kernels                               torch wrappers of every C entry point
"""

from __future__ import annotations

from . import kernels
from .context import reset_runtime_state, routing_context, set_routing_context
from .dense import DenseBackend
from .flex import FlexReuseBackend, FlexReuseConfig
from .spatial import build_spatial_layout

__all__ = [
    "DenseBackend",
    "FlexReuseBackend",
    "FlexReuseConfig",
    "build_spatial_layout",
    "get_backend",
    "kernels",
    "reset_runtime_state",
    "routing_context",
    "set_routing_context",
]

BACKENDS = ("dense", "flex_reuse")


def get_backend(name: str, **config):
    """Backend registry keyed like the reference's ``--backend`` flag (``infer.py:180-223``)."""
    if name == "dense":
        return DenseBackend()
    if name == "flex_reuse":
        return FlexReuseBackend(FlexReuseConfig(**config))
    raise ValueError(f"unknown backend {name!r}; expected one of {BACKENDS}")
