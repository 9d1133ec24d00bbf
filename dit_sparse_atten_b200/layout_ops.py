"""Data-movement ops with the reference's names (``layout_ops.py:86-151``).

``reorder_qkv`` gathers Q/K/V rows through one permutation in one launch and
``pack_boolean_rows`` builds the CSR route; both run the CUDA kernels of
``libbsa.so`` and accept CUDA tensors only.
"""

from __future__ import annotations

import torch

from . import kernels


def reorder_qkv(q, k, v, permutation):
    """Return Q/K/V reordered on axis 1 (``index_select(1, permutation)``)."""
    if not (q.shape == k.shape == v.shape) or q.dim() != 4:
        raise ValueError("q, k and v must share a [B, T, H, D] shape")
    if permutation.dim() != 1 or permutation.numel() != q.shape[1]:
        raise ValueError("permutation must contain one index per token")
    return kernels.reorder_rows([q, k, v], permutation)


def reorder(tensor, permutation):
    """``tensor.index_select(1, permutation)`` for one ``[B, T, ...]`` tensor."""
    return kernels.reorder_rows([tensor], permutation)[0]


def pack_boolean_rows(route):
    """Pack selected column ids first in every row, preserving id order."""
    if route.dtype != torch.bool or route.dim() < 2:
        raise ValueError("route must be a boolean tensor with at least two axes")
    if route.shape[-1] > 4096:
        raise NotImplementedError("at most 4096 columns")
    return kernels.pack_boolean_rows(route)
