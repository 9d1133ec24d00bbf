"""Spatial token layouts for fixed-size route blocks.

* ``build_spatial_layout`` / ``SpatialTokenLayout``: the reference's Morton
  microtile packing (``attention_backends/spatial.py:14-183``).  The
  permutation is host integer work, built once per (grid, block, microtile)
  and cached on each device; the gather itself runs in ``libbsa.so``.
* ``tile_major_layout``: the exact spatial tiles of the reference's sparse
  backend (``attention_backends/sparse.py:51-138``), used with 64-token route
  blocks.

Both layouts expose ``permutation`` (new position -> original token) and its
``inverse``; ``reorder_qkv`` packs and ``restore`` unpacks.
"""

from __future__ import annotations

import math
from collections import Counter, defaultdict
from dataclasses import dataclass, field

import torch

from . import kernels


def _divisors(value):
    return [c for c in range(1, value + 1) if value % c == 0]


def _morton_code(y, x):
    """Interleave coordinate bits, x in the even bits (``spatial.py:19-27``)."""
    result, bit = 0, 0
    while (1 << bit) <= max(y, x):
        result |= ((x >> bit) & 1) << (2 * bit)
        result |= ((y >> bit) & 1) << (2 * bit + 1)
        bit += 1
    return result


def _choose_microtile(height, width, block_size, max_tokens):
    """Largest exact microtile dividing the block, then least elongated."""
    candidates = [(th, tw) for th in _divisors(height) for tw in _divisors(width)
                  if th * tw <= max_tokens and block_size % (th * tw) == 0]
    if not candidates:
        return 1, 1
    return min(candidates, key=lambda s: (-(s[0] * s[1]), abs(math.log(s[1] / s[0]))))


class _DeviceCache:
    def __init__(self):
        self._values = {}

    def get(self, key, build):
        if key not in self._values:
            self._values[key] = build()
        return self._values[key]


@dataclass
class SpatialTokenLayout:
    grid: tuple
    block_size: int
    microtile_shape: tuple
    permutation_cpu: torch.Tensor
    inverse_cpu: torch.Tensor
    neighbors_cpu: torch.Tensor
    block_frames_cpu: torch.Tensor
    _cache: _DeviceCache = field(default_factory=_DeviceCache, repr=False)

    @property
    def tokens(self):
        f, h, w = self.grid
        return f * h * w

    @property
    def blocks(self):
        return math.ceil(self.tokens / self.block_size)

    @property
    def signature(self):
        return self.grid, self.block_size, self.microtile_shape

    def _device_values(self, device):
        device = torch.device(device)
        return self._cache.get(device, lambda: (
            self.permutation_cpu.to(device), self.inverse_cpu.to(device),
            self.neighbors_cpu.to(device)))

    def reorder(self, tensor):
        return kernels.reorder_rows([tensor], self._device_values(tensor.device)[0])[0]

    def reorder_qkv(self, q, k, v):
        """Pack Q/K/V into route-block order with one gather launch."""
        return kernels.reorder_rows([q, k, v], self._device_values(q.device)[0])

    def restore(self, tensor):
        """Unpack an output back to the original (F, H, W) raster order."""
        return kernels.reorder_rows([tensor], self._device_values(tensor.device)[1])[0]

    def neighbors(self, device):
        return self._device_values(device)[2]

    def permutation(self, device):
        """int32 ``[T]`` on ``device``: packed row i holds token ``permutation[i]``
        (also the output rows of the attention's folded unpack)."""
        return self._device_values(device)[0]


def build_spatial_layout(grid, block_size=128, max_microtile_tokens=32):
    """Reversible Morton-ordered packing with no padding (``spatial.py:99-183``)."""
    if grid is None or len(grid) != 3:
        return None
    frames, height, width = (int(v) for v in grid)
    if min(frames, height, width, block_size, max_microtile_tokens) <= 0:
        return None
    th, tw = _choose_microtile(height, width, block_size, max_microtile_tokens)
    tiles_per_block = block_size // (th * tw)
    rows, cols = height // th, width // tw
    frame_order = sorted(((ty, tx) for ty in range(rows) for tx in range(cols)),
                         key=lambda p: (_morton_code(p[0], p[1]), p[0], p[1]))
    ordered = [(f, ty, tx) for f in range(frames) for ty, tx in frame_order]

    # permutation[new] = original token id
    fo = torch.tensor(frame_order, dtype=torch.int64).reshape(-1, 2)
    dy, dx = torch.meshgrid(torch.arange(th), torch.arange(tw), indexing="ij")
    ys = fo[:, 0:1] * th + dy.reshape(1, -1)
    xs = fo[:, 1:2] * tw + dx.reshape(1, -1)
    frame_perm = (ys * width + xs).reshape(-1)
    perm = (torch.arange(frames)[:, None] * (height * width) + frame_perm[None]).reshape(-1)
    permutation = perm.to(torch.int32)
    inverse = torch.empty_like(permutation)
    inverse[permutation.long()] = torch.arange(permutation.numel(), dtype=torch.int32)

    # Route-block neighbours by majority vote over member microtiles.
    tile_block = {}
    block_tiles = defaultdict(list)
    for i, tile in enumerate(ordered):
        tile_block[tile] = i // tiles_per_block
        block_tiles[i // tiles_per_block].append(tile)
    blocks = math.ceil(permutation.numel() / block_size)
    neighbors = torch.full((blocks, 4), -1, dtype=torch.int32)
    block_frames = torch.full((blocks,), -1, dtype=torch.int32)
    for blk in range(blocks):
        tiles = block_tiles[blk]
        frames_in = {t[0] for t in tiles}
        if len(frames_in) == 1:
            block_frames[blk] = next(iter(frames_in))
        for direction, (ddy, ddx) in enumerate(((-1, 0), (1, 0), (0, -1), (0, 1))):
            votes = Counter()
            for f, ty, tx in tiles:
                target = tile_block.get((f, ty + ddy, tx + ddx))
                if target is not None and target != blk:
                    votes[target] += 1
            if votes:
                neighbors[blk, direction] = votes.most_common(1)[0][0]
    return SpatialTokenLayout(grid=(frames, height, width), block_size=block_size,
                              microtile_shape=(th, tw), permutation_cpu=permutation,
                              inverse_cpu=inverse, neighbors_cpu=neighbors,
                              block_frames_cpu=block_frames)


# ----------------------------------------------------------------------------
# Sparse-backend tile-major layout (sparse.py:51-138)
# ----------------------------------------------------------------------------

def _sorted_divisors(value):
    small = [c for c in range(1, math.isqrt(value) + 1) if value % c == 0]
    return small + [value // c for c in reversed(small) if c * c != value]


def sparse_tile_shape(grid, target_tile_tokens):
    """Exact-divisor spatial tile nearest the target (``sparse.py:113-138``)."""
    frames, height, width = (int(v) for v in grid)
    cands = [(a, b) for a in _sorted_divisors(height) for b in _sorted_divisors(width)]
    return min(cands, key=lambda s: (
        abs(math.log((s[0] * s[1]) / target_tile_tokens)) + 0.25 * abs(math.log(s[1] / s[0])),
        abs(s[0] * s[1] - target_tile_tokens),
        -s[0] * s[1]))


@dataclass
class TileMajorLayout:
    """Per-frame (tile_h x tile_w) tiles made contiguous (``sparse.py:81-103``)."""
    grid: tuple
    tile_shape: tuple
    permutation_cpu: torch.Tensor
    inverse_cpu: torch.Tensor
    _cache: _DeviceCache = field(default_factory=_DeviceCache, repr=False)

    @property
    def tile_tokens(self):
        return self.tile_shape[0] * self.tile_shape[1]

    @property
    def signature(self):
        return self.grid, self.tile_shape

    def _device_values(self, device):
        device = torch.device(device)
        return self._cache.get(device, lambda: (self.permutation_cpu.to(device),
                                                self.inverse_cpu.to(device)))

    def reorder_qkv(self, q, k, v):
        return kernels.reorder_rows([q, k, v], self._device_values(q.device)[0])

    def restore(self, tensor):
        return kernels.reorder_rows([tensor], self._device_values(tensor.device)[1])[0]

    def permutation(self, device):
        """int32 ``[T]`` on ``device``: tile-major row i holds token ``permutation[i]``."""
        return self._device_values(device)[0]


def tile_major_layout(grid, tile_h, tile_w):
    frames, height, width = (int(v) for v in grid)
    if height % tile_h or width % tile_w:
        raise ValueError("tile must divide the frame exactly")
    idx = torch.arange(frames * height * width).reshape(
        frames, height // tile_h, tile_h, width // tile_w, tile_w)
    perm = idx.permute(0, 1, 3, 2, 4).reshape(-1).to(torch.int32)
    inverse = torch.empty_like(perm)
    inverse[perm.long()] = torch.arange(perm.numel(), dtype=torch.int32)
    return TileMajorLayout((frames, height, width), (tile_h, tile_w), perm, inverse)
