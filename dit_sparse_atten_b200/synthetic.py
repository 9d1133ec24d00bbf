"""Seeded synthetic workloads for the five configurations of the benchmark.

There is no network and no Wan checkpoint on the build machines, so every input
is generated here from a seed with the shapes, dtypes and value structure the
configurations name.  All generators are deterministic for a given torch
version and device.

* config 1: ``grid=(3, 8, 16)``, 384 tokens, 12 heads, fp32, 8x8 spatial tiles,
  Bernoulli(0.625) route with diagonal and first-frame sink forced on.
* config 2: ``grid=(21, 30, 52)``, 32,760 tokens, CFG batch 2, 12 heads, bf16;
  Q/K RMS-normalised over H*D and 3-D RoPE'd (Wan's published rotary split
  44/42/42 over time/height/width, theta 10000); per-head Gaussian-blob block
  scores (sigma = 3 blocks) for the route.
* config 3: ``grid=(16, 45, 80)``, 57,600 tokens, 40 heads, bf16; Q/K are N(0,1)
  plus a rank-8 smooth spatial field per frame.
* config 4: config 3's grid with CFG batch 2 and 40 heads, Morton-packed, with
  config 2's blob-route procedure over 450 blocks.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LayerConfig:
    name: str
    grid: tuple
    batch: int
    heads: int
    head_dim: int
    block: int = 128
    mass_target: float = 0.95
    keep: float = 0.625

    @property
    def tokens(self):
        return self.grid[0] * self.grid[1] * self.grid[2]

    @property
    def blocks(self):
        return math.ceil(self.tokens / self.block)

    @property
    def sink_blocks(self):
        return math.ceil(self.grid[1] * self.grid[2] / self.block)


CONFIG1 = LayerConfig("config1_cpu_parity", (3, 8, 16), 1, 12, 128, block=64)
CONFIG2 = LayerConfig("config2_wan13b_480p", (21, 30, 52), 2, 12, 128)
CONFIG3 = LayerConfig("config3_route_720p", (16, 45, 80), 1, 40, 128)
CONFIG4 = LayerConfig("config4_wan14b_720p", (16, 45, 80), 2, 40, 128)


def _generator(seed, device):
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


# ----------------------------------------------------------------------------
# config 1
# ----------------------------------------------------------------------------

def config1_inputs(seed=0):
    """q, k, v fp32 ``[1, 384, 12, 128]`` and the route ``[12, 6, 6]`` (CPU).

    Draw order from one ``torch.Generator`` seeded with ``seed``: q, k, v
    (``randn / sqrt(128)``), then ``rand(12, 6, 6) < 0.625``; the diagonal and
    the first frame's two tiles (key blocks 0 and 1) are then forced on.
    """
    c = CONFIG1
    g = _generator(seed, "cpu")
    shape = (1, c.tokens, c.heads, c.head_dim)
    q = torch.randn(shape, generator=g) / math.sqrt(c.head_dim)
    k = torch.randn(shape, generator=g) / math.sqrt(c.head_dim)
    v = torch.randn(shape, generator=g) / math.sqrt(c.head_dim)
    blocks = c.tokens // c.block
    route = torch.rand((c.heads, blocks, blocks), generator=g) < 0.625
    route |= torch.eye(blocks, dtype=torch.bool)
    sink = (c.grid[1] * c.grid[2]) // c.block
    route[..., :sink] = True
    return q, k, v, route


# ----------------------------------------------------------------------------
# Wan-style Q/K preparation (config 2)
# ----------------------------------------------------------------------------

def rms_norm(x, eps=1e-6):
    """RMSNorm over the flattened H*D features with unit weight."""
    shape = x.shape
    flat = x.reshape(shape[0], shape[1], -1).float()
    flat = flat * torch.rsqrt(flat.pow(2).mean(-1, keepdim=True) + eps)
    return flat.reshape(shape)


def rope_3d(x, grid, theta=10000.0):
    """Apply Wan's 3-D rotary embedding to ``[B, T, H, D]`` in (F, H, W) order.

    The head dimension is split into complex pairs for time, height and width
    with ``D - 4*(D//6)``, ``2*(D//6)``, ``2*(D//6)`` real channels; pair ``j``
    of an axis with ``n`` channels rotates by ``pos * theta**(-2j/n)``.
    """
    frames, height, width = grid
    dim = x.shape[-1]
    parts = (dim - 4 * (dim // 6), 2 * (dim // 6), 2 * (dim // 6))
    device = x.device
    angles = []
    positions = torch.stack(torch.meshgrid(
        torch.arange(frames, device=device), torch.arange(height, device=device),
        torch.arange(width, device=device), indexing="ij"), -1).reshape(-1, 3).double()
    for axis, n in enumerate(parts):
        inv = theta ** (-torch.arange(0, n, 2, device=device, dtype=torch.float64) / n)
        angles.append(positions[:, axis:axis + 1] * inv[None])
    ang = torch.cat(angles, -1)                      # [T, D/2]
    cos = ang.cos().float()[None, :, None, :]
    sin = ang.sin().float()[None, :, None, :]
    xf = x.float().reshape(*x.shape[:-1], dim // 2, 2)
    re, im = xf[..., 0], xf[..., 1]
    out = torch.stack((re * cos - im * sin, re * sin + im * cos), -1)
    return out.reshape(x.shape)


def prologue_inputs(batch, grid, heads, head_dim=128, seed=0):
    """Seeded inputs of the attention prologue: bf16 projections
    ``[B, T, H*D]`` (scaled so that the norm matters), bf16 RMSNorm weights
    ``[H*D]`` and the complex rotary table ``[T, D/2]`` of Wan's 3-D RoPE
    (``rope_3d``'s angles)."""
    g = _generator(seed, "cpu")
    frames, height, width = grid
    T, C = frames * height * width, heads * head_dim
    proj = [(torch.randn((batch, T, C), generator=g) * 2.5).to(torch.bfloat16) for _ in range(3)]
    weights = [(torch.rand(C, generator=g) + 0.5).to(torch.bfloat16) for _ in range(2)]
    parts = (head_dim - 4 * (head_dim // 6), 2 * (head_dim // 6), 2 * (head_dim // 6))
    positions = torch.stack(torch.meshgrid(torch.arange(frames), torch.arange(height),
                                           torch.arange(width), indexing="ij"), -1).reshape(-1, 3)
    angles = []
    for axis, n in enumerate(parts):
        inv = 10000.0 ** (-torch.arange(0, n, 2, dtype=torch.float64) / n)
        angles.append(positions[:, axis:axis + 1].double() * inv[None])
    ang = torch.cat(angles, -1)
    rotary = torch.polar(torch.ones_like(ang), ang).to(torch.complex64)
    return proj, weights, rotary


def wan_qkv(config, seed=0, device="cpu", dtype=torch.bfloat16):
    """q, k, v ``[B, T, H, D]``: RMS-normalised + 3-D RoPE'd Q/K, N(0,1) V."""
    g = _generator(seed, device)
    shape = (config.batch, config.tokens, config.heads, config.head_dim)
    q = torch.randn(shape, generator=g, device=device)
    k = torch.randn(shape, generator=g, device=device)
    v = torch.randn(shape, generator=g, device=device)
    q = rope_3d(rms_norm(q), config.grid)
    k = rope_3d(rms_norm(k), config.grid)
    return q.to(dtype), k.to(dtype), v.to(dtype)


# ----------------------------------------------------------------------------
# Gaussian-blob block scores (configs 2 and 4)
# ----------------------------------------------------------------------------

def blob_scores(heads, blocks, seed=0, sigma=3.0, blobs=8, device="cpu"):
    """Per-head spatially smooth block mass ``[H, Qb, Kb]`` (rows sum to 1).

    Each head gets ``blobs`` Gaussian bumps (sigma in blocks) at seeded
    (query-block, key-block) centres with U(0.5, 1.5) amplitude, a diagonal
    band of the same width, and a U(0, 0.02) floor; rows are normalised.
    """
    g = _generator(seed, device)
    idx = torch.arange(blocks, device=device, dtype=torch.float32)
    qi = idx[:, None]
    ki = idx[None, :]
    out = torch.empty((heads, blocks, blocks), device=device)
    for h in range(heads):
        centres = torch.rand((blobs, 2), generator=g, device=device) * blocks
        amps = 0.5 + torch.rand((blobs,), generator=g, device=device)
        score = torch.exp(-((qi - ki) ** 2) / (2 * sigma ** 2))
        for b in range(blobs):
            score = score + amps[b] * torch.exp(
                -((qi - centres[b, 0]) ** 2 + (ki - centres[b, 1]) ** 2) / (2 * sigma ** 2))
        score = score + 0.02 * torch.rand((blocks, blocks), generator=g, device=device)
        out[h] = score / score.sum(-1, keepdim=True)
    return out


# ----------------------------------------------------------------------------
# config 3: N(0,1) + rank-8 per-frame spatial structure
# ----------------------------------------------------------------------------

def structured_qk(config, seed=0, device="cpu", dtype=torch.bfloat16, rank=8, strength=2.0):
    """q, k ``[B, T, H, D]``: N(0,1) noise plus a rank-``rank`` smooth spatial field.

    For frame f, basis function r is ``cos(2*pi*(a_r*y/H + b_r*x/W) + phase_{f,r})``
    with integer frequencies a_r, b_r in [0, 2]; Q's loadings are N(0,1) per
    (frame, head, r), K's are Q's plus 0.5*N(0,1).
    """
    g = _generator(seed, device)
    frames, height, width = config.grid
    B, H, D = config.batch, config.heads, config.head_dim
    shape = (B, config.tokens, H, D)
    q = torch.randn(shape, generator=g, device=device)
    k = torch.randn(shape, generator=g, device=device)
    freq = torch.randint(0, 3, (rank, 2), generator=g, device=device).float()
    phase = torch.rand((frames, rank), generator=g, device=device) * 2 * math.pi
    load_q = torch.randn((frames, H, rank, D), generator=g, device=device)
    load_k = load_q + 0.5 * torch.randn((frames, H, rank, D), generator=g, device=device)
    yy, xx = torch.meshgrid(torch.arange(height, device=device) / height,
                            torch.arange(width, device=device) / width, indexing="ij")
    coord = 2 * math.pi * (freq[:, 0, None, None] * yy + freq[:, 1, None, None] * xx)  # [r,Hg,Wg]
    basis = torch.cos(coord[None] + phase[:, :, None, None])                             # [F,r,Hg,Wg]
    basis = basis.reshape(frames, rank, height * width)
    fq = torch.einsum("frt,fhrd->fthd", basis, load_q).reshape(1, config.tokens, H, D)
    fk = torch.einsum("frt,fhrd->fthd", basis, load_k).reshape(1, config.tokens, H, D)
    amp = strength / math.sqrt(rank)
    return (q + amp * fq).to(dtype), (k + amp * fk).to(dtype)


def previous_route(heads, blocks, seed=0, density=0.6, device="cpu"):
    """Seeded previous route ``[H, Qb, Kb]`` for the persistence prior."""
    g = _generator(seed, device)
    return torch.rand((heads, blocks, blocks), generator=g, device=device) < density
