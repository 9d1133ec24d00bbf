"""Block-sparse attention restated in numpy (test oracle; see ``oracle/__init__``).

Semantics follow the reference's sparse reference backend ``sparse_chunk``
(``attention_backends/sparse.py:670-751``: per (query tile, head) gather of the
selected key tiles, masked softmax, PV) and FlexAttention's full-block route
(``attention_backends/flex.py:308-355,379-399``: a query in block ``qb`` of head
``h`` attends to every valid key ``< T`` in the key blocks selected by
``route[h, qb]``).
"""

from __future__ import annotations

import math

import numpy as np


def block_sparse_attention(q, k, v, route, block, scale=None, query_blocks=None,
                           dtype=np.float64, return_lse=False):
    """Attention for one batch element.

    ``q``/``k``/``v``: ``[T, H, D]``; ``route``: bool ``[H, Qb, Kb]``.
    ``query_blocks`` optionally restricts the computed query blocks (other rows
    are left as NaN).  Rows with an empty route are zero (the CUDA kernel's
    documented convention; the reference never produces them).
    """
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    route = np.asarray(route, bool)
    tokens, heads, dim = q.shape
    blocks = math.ceil(tokens / block)
    if route.shape != (heads, blocks, blocks):
        raise ValueError(f"route shape {route.shape} != {(heads, blocks, blocks)}")
    s = scale if scale is not None else dim ** -0.5
    out = np.full((tokens, heads, v.shape[-1]), np.nan, dtype)
    lse = np.full((heads, tokens), np.nan, dtype)
    qbs = range(blocks) if query_blocks is None else query_blocks
    token_block = np.arange(tokens) // block
    for h in range(heads):
        for qb in qbs:
            rows = slice(qb * block, min(tokens, (qb + 1) * block))
            keys = np.nonzero(route[h, qb][token_block])[0]
            if keys.size == 0:
                out[rows, h] = 0
                lse[h, rows] = -np.inf
                continue
            scores = q[rows, h] @ k[keys, h].T * s
            m = scores.max(-1, keepdims=True)
            e = np.exp(scores - m)
            l = e.sum(-1, keepdims=True)
            out[rows, h] = (e / l) @ v[keys, h]
            lse[h, rows] = (m + np.log(l))[:, 0]
    return (out, lse) if return_lse else out


def dense_masked_attention(q, k, v, route, block, scale=None):
    """Explicit masked softmax over all keys (``tests/test_flex_backend.py:138-148``)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    tokens, heads, dim = q.shape
    s = scale if scale is not None else dim ** -0.5
    ids = np.arange(tokens) // block
    out = np.empty((tokens, heads, v.shape[-1]))
    for h in range(heads):
        allowed = np.asarray(route, bool)[h][ids[:, None], ids[None, :]]
        scores = np.where(allowed, q[:, h] @ k[:, h].T * s, -np.inf)
        scores = scores - scores.max(-1, keepdims=True)
        p = np.exp(scores)
        out[:, h] = (p / p.sum(-1, keepdims=True)) @ v[:, h]
    return out


def kept_block_flops(route_counts_or_route, tokens, block, dim):
    """Algorithmic FLOPs of QK^T + PV over kept blocks: ``4 * q_valid * k_valid * D``."""
    route = np.asarray(route_counts_or_route, bool)
    blocks = route.shape[-1]
    sizes = np.minimum(tokens - np.arange(blocks) * block, block).astype(np.float64)
    per = sizes[:, None] * sizes[None, :]
    return float(4.0 * dim * (route * per).sum())
