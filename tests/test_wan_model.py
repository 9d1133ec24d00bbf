"""The config-5 transformer forward (``dit_sparse_atten_b200/wan_model.py``) on CPU.

A tiny Wan configuration (2 layers, dim 64, 4 heads of 16) runs the 5-step
denoising loop in one process, then on two gloo ranks in both layouts the GPU
run uses: CFG branches on separate ranks, and one branch's tokens split over
two ranks with the self-attention exchanged head-parallel.  Every layout must
give the single-process latents (float32, summation order aside).  The
self-attention here is dense SDPA and the Q/K prologue a torch restatement:
the routed kernels themselves are CUDA-only and covered by the GPU tests.
Reference structure: ``attention_backends/wan_diffusers.py:75-191``.
"""

import math

import torch
import torch.distributed as dist

from dit_sparse_atten_b200 import parallel, wan_model
from test_parallel_gloo import CpuRows, run_ranks

TINY = wan_model.WanConfig(dim=64, ffn=96, heads=4, layers=2, in_channels=4, out_channels=4,
                           text_dim=24, text_tokens=8, freq_dim=16)
GRID = (2, 4, 8)          # 64 tokens after the 1x2x2 patch
STEPS = 3


def torch_prologue(heads, eps):
    """RMSNorm of Q and K over dim (block weights), then the rotary embedding."""
    def run(q, k, v, blk, cos, sin):
        t = q.shape[0]

        def norm(x, w):
            xf = x.float()
            return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()

        def rope(x):
            x = x.view(t, heads, -1, 2)
            re, im = x[..., 0], x[..., 1]
            c, s = cos[:, None], sin[:, None]
            return torch.stack((re * c - im * s, re * s + im * c), -1).view(t, heads, -1)

        return (rope(norm(q, blk["norm_q"])).to(q.dtype)[None],
                rope(norm(k, blk["norm_k"])).to(k.dtype)[None],
                v.view(t, heads, -1)[None])
    return run


def sdpa(q, k, v):
    o = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                                         v.transpose(1, 2))
    return o.transpose(1, 2)


def inputs():
    g = torch.Generator().manual_seed(3)
    frames, h, w = GRID
    latent = torch.randn((TINY.in_channels, frames, 2 * h, 2 * w), generator=g)
    text = [torch.randn((1, TINY.text_tokens, TINY.text_dim), generator=g) for _ in range(2)]
    return wan_model.patchify(latent, TINY), text


def generate(branches, shard, combine):
    weights = wan_model.WanWeights(TINY, "cpu", seed=1, dtype=torch.float32)
    model = wan_model.WanTransformer(weights, GRID, shard, torch_prologue(TINY.heads, TINY.eps))
    patches, text = inputs()
    rows = patches[model.rows]
    contexts = {b: model.context(text[b]) for b in branches}

    def attention(q, k, v):
        return parallel.head_parallel_attention(q, k, v, sdpa, shard.group, shard.size,
                                                rows=CpuRows)

    return wan_model.denoise(model, rows, contexts, attention, combine, steps=STEPS)


def single_process():
    return generate([0, 1], wan_model.SequenceShard(), wan_model.CfgCombine(5.0))


def test_shapes_and_single_process_run():
    out = single_process()
    frames, h, w = GRID
    assert out.shape == (math.prod(GRID), TINY.in_channels * 4)
    assert torch.isfinite(out).all()
    weights = wan_model.WanWeights(TINY, "cpu", seed=1, dtype=torch.float32)
    per_block = 4 * (64 * 64 + 64) * 2 + 2 * 64 * 96 + 96 + 64 + 6 * 64 + 6 * 64
    assert weights.parameter_count() > TINY.layers * per_block


def test_14b_shapes():
    cfg = wan_model.WAN_14B
    assert (cfg.dim, cfg.ffn, cfg.heads, cfg.layers, cfg.head_dim) == (5120, 13824, 40, 40, 128)
    cos, sin = wan_model.rotary_tables(cfg, (16, 45, 80))
    assert cos.shape == (57600, 64) and sin.shape == (57600, 64)
    sig = wan_model.flow_sigmas(5)
    assert sig[0] == 1.0 and sig[-1] == 0.0 and all(a > b for a, b in zip(sig, sig[1:]))


def _cfg_split(rank, world):
    # one branch per rank, all tokens local: the pair group is the world
    shard = wan_model.SequenceShard()
    combine = wan_model.CfgCombine(5.0, pair_group=dist.group.WORLD)
    return generate([rank], shard, combine).numpy()   # numpy: pickled by value


def _sequence_split(rank, world):
    # both branches per rank, tokens split over the two ranks
    shard = wan_model.SequenceShard(dist.group.WORLD, world, rank)
    return generate([0, 1], shard, wan_model.CfgCombine(5.0)).numpy()


def test_cfg_branches_on_two_ranks_match_one_process():
    ref = single_process()
    results = run_ranks(_cfg_split, world=2)
    for rank in range(2):
        torch.testing.assert_close(torch.from_numpy(results[rank]), ref, atol=1e-4, rtol=1e-4)


def test_sequence_parallel_matches_one_process():
    ref = single_process()
    results = run_ranks(_sequence_split, world=2)
    t = ref.shape[0] // 2
    for rank in range(2):
        torch.testing.assert_close(torch.from_numpy(results[rank]), ref[rank * t:(rank + 1) * t],
                                   atol=1e-4, rtol=1e-4)
