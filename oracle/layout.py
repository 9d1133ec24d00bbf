"""Spatial token permutations restated in numpy (test oracle; see ``oracle/__init__``).

* ``morton_layout``: the Morton microtile packing of
  ``attention_backends/spatial.py:99-183`` (permutation and inverse only).
* ``tile_major_layout``: the sparse reference backend's exact spatial tiles
  (``attention_backends/sparse.py:81-92,113-138``).
* ``reorder``: ``tensor.index_select(1, permutation)`` (``spatial.py:82-93``).
"""

from __future__ import annotations

import math

import numpy as np


def morton_code(y: int, x: int) -> int:
    """Bit interleave, x in even bits (``spatial.py:19-27``)."""
    code, bit = 0, 0
    while (1 << bit) <= max(y, x):
        code |= ((x >> bit) & 1) << (2 * bit)
        code |= ((y >> bit) & 1) << (2 * bit + 1)
        bit += 1
    return code


def choose_microtile(height, width, block, max_tokens):
    """Largest exact microtile, then least elongated (``spatial.py:30-43``)."""
    best = None
    for th in range(1, height + 1):
        if height % th:
            continue
        for tw in range(1, width + 1):
            if width % tw:
                continue
            area = th * tw
            if area <= max_tokens and block % area == 0:
                key = (-area, abs(math.log(tw / th)))
                if best is None or key < best[0]:
                    best = (key, (th, tw))
    return (1, 1) if best is None else best[1]


def morton_layout(grid, block=128, max_microtile_tokens=32):
    frames, height, width = grid
    th, tw = choose_microtile(height, width, block, max_microtile_tokens)
    rows, cols = height // th, width // tw
    tiles = sorted(((ty, tx) for ty in range(rows) for tx in range(cols)),
                   key=lambda p: (morton_code(p[0], p[1]), p[0], p[1]))
    ty = np.array([t[0] for t in tiles])
    tx = np.array([t[1] for t in tiles])
    dy, dx = np.meshgrid(np.arange(th), np.arange(tw), indexing="ij")
    ys = ty[:, None] * th + dy.reshape(1, -1)
    xs = tx[:, None] * tw + dx.reshape(1, -1)
    frame_perm = (ys * width + xs).reshape(-1)
    perm = (np.arange(frames)[:, None] * height * width + frame_perm[None]).reshape(-1)
    perm = perm.astype(np.int32)
    inverse = np.empty_like(perm)
    inverse[perm] = np.arange(perm.size, dtype=np.int32)
    return (th, tw), perm, inverse


def sparse_tile_shape(grid, target_tile_tokens):
    """Exact-divisor spatial tile nearest the target (``sparse.py:113-138``)."""
    frames, height, width = grid

    def divisors(v):
        small = [c for c in range(1, math.isqrt(v) + 1) if v % c == 0]
        return small + [v // c for c in reversed(small) if c * c != v]

    cands = [(a, b) for a in divisors(height) for b in divisors(width)]
    return min(cands, key=lambda s: (
        abs(math.log((s[0] * s[1]) / target_tile_tokens)) + 0.25 * abs(math.log(s[1] / s[0])),
        abs(s[0] * s[1] - target_tile_tokens),
        -s[0] * s[1],
    ))


def tile_major_layout(grid, tile_h, tile_w):
    """Permutation that makes each (tile_h x tile_w) spatial tile contiguous."""
    frames, height, width = grid
    idx = np.arange(frames * height * width).reshape(
        frames, height // tile_h, tile_h, width // tile_w, tile_w)
    perm = idx.transpose(0, 1, 3, 2, 4).reshape(-1).astype(np.int32)
    inverse = np.empty_like(perm)
    inverse[perm] = np.arange(perm.size, dtype=np.int32)
    return perm, inverse


def reorder(x, perm):
    """``x.index_select(1, perm)`` for ``[B, T, ...]`` arrays."""
    return np.asarray(x)[:, np.asarray(perm, np.int64)]
