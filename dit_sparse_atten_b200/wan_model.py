"""Wan2.1 text-to-video transformer forward for the 5-step measurement (config 5).

The reference drives Diffusers' ``WanTransformer3DModel`` through its own
frontend: ``_model_forward`` (``attention_backends/wan_diffusers.py:120-191``:
patch embedding, time/text conditioning, the rotary table of the (F, H, W)
grid, 40 blocks, output norm and projection) and ``_block_forward``
(``wan_diffusers.py:75-117``: modulated LayerNorm -> self-attention through
the backend -> gated residual; LayerNorm -> text cross-attention; modulated
LayerNorm -> GELU FFN -> gated residual), with ``StudyWanProcessor``
(``wan_diffusers.py:21-70``) for the self-attention.  ``infer.py:226-285``
runs it inside the Diffusers pipeline: per denoising step one transformer
call per CFG branch, then the scheduler step.

This module restates that forward with random-init weights (no checkpoint on
these machines) for timing on 1-8 GPUs:

* sequence parallel: a rank holds ``T/P`` tokens of its CFG branch for every
  per-token op (projections, norms, FFN, cross-attention, the scheduler step),
  and the self-attention runs head-parallel behind a sequence<->head
  all-to-all (``parallel.head_parallel_attention``);
* CFG branches on two rank groups when the world size is even (cond on group
  0, uncond on group 1), joined per step by one all-reduce of the weighted
  noise predictions over the two ranks that hold the same tokens;
* the Q/K RMSNorm + RoPE run as the fused prologue kernel on CUDA
  (``kernels.qkv_prologue``, without the reorder: the permutation spans all
  tokens, so the backend packs after the exchange);
* every other op is PyTorch (cuBLAS GEMMs, library SDPA for the 512-token
  cross-attention).

Weights: ``nn.Linear``'s default uniform(+-1/sqrt(fan_in)) for every
projection, modulation tables N(0, 1/dim), norm weights 1 + U(-0.1, 0.1),
seeded; the Wan2.1-14B shapes (dim 5120, FFN 13824, 40 heads, 40 layers,
text 512 x 4096, patch 1x2x2, 16 latent channels).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .context import set_routing_context


@dataclass(frozen=True)
class WanConfig:
    dim: int = 5120
    ffn: int = 13824
    heads: int = 40
    layers: int = 40
    in_channels: int = 16
    out_channels: int = 16
    text_dim: int = 4096
    text_tokens: int = 512
    freq_dim: int = 256
    patch: tuple = (1, 2, 2)
    eps: float = 1e-6
    theta: float = 10000.0

    @property
    def head_dim(self):
        return self.dim // self.heads

    @property
    def patch_size(self):
        return self.patch[0] * self.patch[1] * self.patch[2]


WAN_14B = WanConfig()


def _uniform(shape, fan_in, gen, device):
    bound = 1.0 / math.sqrt(fan_in)
    return (torch.rand(shape, generator=gen, device=device) * 2 - 1) * bound


class WanWeights:
    """Random-init weights of one Wan transformer (bf16 on ``device``)."""

    def __init__(self, cfg: WanConfig, device, seed=0, dtype=torch.bfloat16):
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        d, dt = cfg.dim, dtype

        def linear(out_f, in_f):
            return (_uniform((out_f, in_f), in_f, g, device).to(dt),
                    _uniform((out_f,), in_f, g, device).to(dt))

        def norm_weight(n):
            return (1 + (torch.rand((n,), generator=g, device=device) - 0.5) * 0.2).to(dt)

        self.cfg = cfg
        self.patch = linear(d, cfg.in_channels * cfg.patch_size)
        self.time_1 = linear(d, cfg.freq_dim)
        self.time_2 = linear(d, d)
        self.time_proj = linear(6 * d, d)
        self.text_1 = linear(d, cfg.text_dim)
        self.text_2 = linear(d, d)
        self.blocks = []
        for _ in range(cfg.layers):
            blk = {
                "table": torch.randn((1, 6, d), generator=g, device=device) / math.sqrt(d),
                "q": linear(d, d), "k": linear(d, d), "v": linear(d, d), "o": linear(d, d),
                "norm_q": norm_weight(d), "norm_k": norm_weight(d),
                "norm2_w": norm_weight(d), "norm2_b": torch.zeros((d,), device=device, dtype=dt),
                "q2": linear(d, d), "k2": linear(d, d), "v2": linear(d, d), "o2": linear(d, d),
                "norm_q2": norm_weight(d), "norm_k2": norm_weight(d),
                "ffn1": linear(cfg.ffn, d), "ffn2": linear(d, cfg.ffn),
            }
            self.blocks.append(blk)
        self.out_table = torch.randn((1, 2, d), generator=g, device=device) / math.sqrt(d)
        self.proj_out = linear(cfg.out_channels * cfg.patch_size, d)

    def parameter_count(self):
        total = sum(w.numel() + b.numel() for w, b in (self.patch, self.time_1, self.time_2,
                                                       self.time_proj, self.text_1, self.text_2,
                                                       self.proj_out))
        for blk in self.blocks:
            for v in blk.values():
                total += sum(t.numel() for t in v) if isinstance(v, tuple) else v.numel()
        return total


def rotary_tables(cfg: WanConfig, grid):
    """Wan's 3-D rotary table for an (F, H, W) token grid: ``(cos, sin)`` fp32
    ``[T, D/2]``; the head dimension splits into time/height/width pairs as
    ``D - 4*(D//6)``, ``2*(D//6)``, ``2*(D//6)`` channels and pair j of an
    axis with n channels turns by ``pos * theta**(-2j/n)`` (Wan's published
    rotary embedding, float64 angles)."""
    frames, height, width = grid
    dim = cfg.head_dim
    parts = (dim - 4 * (dim // 6), 2 * (dim // 6), 2 * (dim // 6))
    pos = torch.stack(torch.meshgrid(torch.arange(frames), torch.arange(height),
                                     torch.arange(width), indexing="ij"), -1).reshape(-1, 3)
    angles = []
    for axis, n in enumerate(parts):
        inv = cfg.theta ** (-torch.arange(0, n, 2, dtype=torch.float64) / n)
        angles.append(pos[:, axis:axis + 1].double() * inv[None])
    ang = torch.cat(angles, -1)
    return ang.cos().float(), ang.sin().float()


def timestep_embedding(t, dim):
    """Sinusoidal embedding of a scalar timestep: ``[cos(t f_i), sin(t f_i)]``
    with ``f_i = 10000^(-i / (dim/2))``."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32) / half)
    arg = float(t) * freqs
    return torch.cat([arg.cos(), arg.sin()])[None]


def patchify(latent, cfg: WanConfig):
    """``[C, F, H, W]`` latent -> ``[F * H/2 * W/2, C * 4]`` patch rows (token
    order f, y, x; features c, py, px as Conv3d with a 1x2x2 kernel flattens
    its weight)."""
    c, f, h, w = latent.shape
    pf, ph, pw = cfg.patch
    x = latent.reshape(c, f // pf, pf, h // ph, ph, w // pw, pw)
    x = x.permute(1, 3, 5, 0, 2, 4, 6)
    return x.reshape((f // pf) * (h // ph) * (w // pw), c * pf * ph * pw)


@dataclass
class SequenceShard:
    """This rank's place in the sequence-parallel layout of one CFG branch."""
    group: object = None      # process group of the ranks sharing the branch
    size: int = 1             # ranks in that group (the all-to-all width)
    index: int = 0            # this rank's token shard


def _linear(x, wb):
    return F.linear(x, wb[0], wb[1])


def _rms(x, weight, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * weight


class WanTransformer:
    """One CFG branch's transformer forward on this rank's token shard.

    ``attention(q, k, v)`` computes the self-attention of ``[1, T/P, H, D]``
    shards (head-parallel exchange + a backend); ``prologue(q, k, v, block,
    cos, sin)`` turns ``[T/P, dim]`` projections into normalised, rotated
    ``[1, T/P, H, D]`` tensors (the fused kernel on CUDA).
    """

    def __init__(self, weights: WanWeights, grid, shard: SequenceShard, prologue):
        self.w = weights
        self.cfg = weights.cfg
        self.grid = tuple(grid)
        self.shard = shard
        self.prologue = prologue
        tokens = math.prod(self.grid)
        if tokens % shard.size:
            raise ValueError(f"{tokens} tokens do not split over {shard.size} ranks")
        self.tokens_local = tokens // shard.size
        rows = slice(shard.index * self.tokens_local, (shard.index + 1) * self.tokens_local)
        cos, sin = rotary_tables(self.cfg, self.grid)
        device = weights.patch[0].device
        self.rope = (cos[rows].contiguous().to(device), sin[rows].contiguous().to(device))
        self.rows = rows

    def context(self, text):
        """Text conditioning ``[1, 512, text_dim]`` -> ``[1, 512, dim]`` (once per
        generation: the reference's condition embedder)."""
        h = F.gelu(_linear(text, self.w.text_1), approximate="tanh")
        return _linear(h, self.w.text_2)

    def forward(self, patches, t, ctx, attention, step, branch):
        """Noise prediction ``[T/P, out * 4]`` for this rank's ``patches``
        ``[T/P, C * 4]`` at timestep ``t`` (``wan_diffusers.py:120-191``)."""
        cfg, w = self.cfg, self.w
        dtype = w.patch[0].dtype
        device = patches.device
        x = _linear(patches.to(dtype), w.patch)[None]                    # [1, T/P, dim]
        emb = timestep_embedding(t, cfg.freq_dim).to(device, dtype)
        temb = _linear(F.silu(_linear(emb, w.time_1)), w.time_2)         # [1, dim]
        tproj = _linear(F.silu(temb), w.time_proj).unflatten(1, (6, cfg.dim))
        for layer, blk in enumerate(w.blocks):
            set_routing_context(attention_id=layer, step=step, branch=branch, grid=self.grid)
            x = self._block(x, blk, ctx, tproj, attention)
        shift, scale = (w.out_table + temb.float()[:, None]).chunk(2, dim=1)
        h = F.layer_norm(x.float(), (cfg.dim,), eps=cfg.eps) * (1 + scale) + shift
        return _linear(h.to(dtype), w.proj_out)[0]

    def _block(self, x, blk, ctx, tproj, attention):
        cfg = self.cfg
        dtype = x.dtype
        shift, scale, gate, c_shift, c_scale, c_gate = (blk["table"] + tproj.float()).chunk(6, 1)
        # self-attention (StudyWanProcessor: projections, prologue, backend, to_out)
        h = (F.layer_norm(x.float(), (cfg.dim,), eps=cfg.eps) * (1 + scale) + shift).to(dtype)
        q, k, v = _linear(h[0], blk["q"]), _linear(h[0], blk["k"]), _linear(h[0], blk["v"])
        q, k, v = self.prologue(q, k, v, blk, *self.rope)
        a = attention(q, k, v).flatten(2, 3)
        x = (x.float() + _linear(a, blk["o"]).float() * gate).to(dtype)
        # text cross-attention (dense library SDPA over the 512 text tokens)
        h = F.layer_norm(x.float(), (cfg.dim,), blk["norm2_w"].float(), blk["norm2_b"].float(),
                         cfg.eps).to(dtype)
        heads, hd = cfg.heads, cfg.head_dim
        q2 = _rms(_linear(h, blk["q2"]), blk["norm_q2"], cfg.eps).unflatten(2, (heads, hd))
        k2 = _rms(_linear(ctx, blk["k2"]), blk["norm_k2"], cfg.eps).unflatten(2, (heads, hd))
        v2 = _linear(ctx, blk["v2"]).unflatten(2, (heads, hd))
        a2 = F.scaled_dot_product_attention(q2.transpose(1, 2), k2.transpose(1, 2),
                                            v2.transpose(1, 2)).transpose(1, 2).flatten(2, 3)
        x = x + _linear(a2, blk["o2"])
        # feed-forward
        h = (F.layer_norm(x.float(), (cfg.dim,), eps=cfg.eps) * (1 + c_scale) + c_shift).to(dtype)
        f = _linear(F.gelu(_linear(h, blk["ffn1"]), approximate="tanh"), blk["ffn2"])
        return (x.float() + f.float() * c_gate).to(dtype)


def fused_prologue(heads, eps):
    """The CUDA prologue (``kernels.qkv_prologue``): RMSNorm of Q and K over
    ``dim`` with the block's weights and the rotary embedding, one pass, no
    reorder (the sequence is sharded; the backend packs after the exchange)."""
    from . import kernels

    def run(q, k, v, blk, cos, sin):
        return kernels.qkv_prologue(q[None], k[None], v[None], heads,
                                    norm_q_weight=blk["norm_q"], norm_k_weight=blk["norm_k"],
                                    eps=eps, rope_cos=cos, rope_sin=sin)
    return run


def flow_sigmas(steps, shift=5.0):
    """Flow-matching noise levels of a ``steps``-step run with Wan's shift:
    ``s' = shift * s / (1 + (shift - 1) * s)`` over ``s = 1 .. 0``."""
    s = torch.linspace(1.0, 0.0, steps + 1, dtype=torch.float64)
    return (shift * s / (1 + (shift - 1) * s)).tolist()


class CfgCombine:
    """Classifier-free guidance across ranks: ``uncond + g * (cond - uncond)``.

    With the branches on two rank groups, the two ranks that hold the same
    tokens (one per group) sum ``g * cond`` and ``(1 - g) * uncond`` with one
    all-reduce over their pair group; with both branches on this rank the sum
    is local.  Branch 0 is the conditional call, branch 1 the unconditional
    one (the reference counts the repeated timestep as branch 1).
    """

    def __init__(self, guidance, pair_group=None):
        self.guidance = guidance
        self.pair_group = pair_group

    def weight(self, branch):
        return self.guidance if branch == 0 else 1.0 - self.guidance

    def __call__(self, preds):
        total = None
        for branch, pred in preds.items():
            part = pred.float() * self.weight(branch)
            total = part if total is None else total + part
        if self.pair_group is not None:
            import torch.distributed as dist
            dist.all_reduce(total, group=self.pair_group)
        return total


def denoise(model: WanTransformer, patches, contexts, attention, combine, steps=5, shift=5.0,
            on_step=None):
    """``steps`` flow-matching Euler steps on this rank's latent patch rows
    ``[T/P, C * 4]``: per step one transformer call per CFG branch this rank
    owns (``contexts``: branch -> text context), the guidance combination,
    ``x += (sigma_next - sigma) * v``.  Returns the final rows (float32)."""
    sigmas = flow_sigmas(steps, shift)
    x = patches.float()
    for i in range(steps):
        t = sigmas[i] * 1000.0
        preds = {b: model.forward(x, t, ctx, attention, i, b) for b, ctx in contexts.items()}
        v = combine(preds)
        x = x + (sigmas[i + 1] - sigmas[i]) * v
        if on_step is not None:
            on_step(i)
    return x


def pair_groups(world, group_size):
    """Process groups {r, r + group_size} (the two ranks that hold token shard
    r, one per CFG branch); every rank creates all of them in the same order.
    Returns this rank's group."""
    import torch.distributed as dist
    mine = None
    rank = dist.get_rank()
    for r in range(group_size):
        pg = dist.new_group([r, r + group_size])
        if rank in (r, r + group_size):
            mine = pg
    return mine
