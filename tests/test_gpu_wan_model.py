"""The config-5 frontend on the GPU with the routed kernels.

A 2-layer Wan model with head_dim 128 (dim 256, 2 heads) on a (2, 16, 32)
token grid runs three denoising steps through ``FlexReuseBackend`` with the
spatial reorder and the fused prologue kernel.  With keep 1 and mass target 1
every route keeps every block, so after the dense step 0 and layer 0 the
sparse kernels compute full attention and the result must match the same
generation with dense SDPA attention (bf16 tolerance).  A second run with the
reference's recommended flags checks the phase bookkeeping over the steps.
Reference structure: ``attention_backends/wan_diffusers.py:75-191``.
"""

import pytest
import torch

from dit_sparse_atten_b200 import _native, parallel, wan_model
from dit_sparse_atten_b200.context import reset_runtime_state
from dit_sparse_atten_b200.dense import DenseBackend
from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig

pytestmark = pytest.mark.gpu

CFG = wan_model.WanConfig(dim=256, ffn=512, heads=2, layers=2, in_channels=4, out_channels=4,
                          text_dim=64, text_tokens=16, freq_dim=32)
GRID = (2, 16, 32)        # 1,024 tokens, 8 route blocks
STEPS = 3


def generate(backend):
    device = torch.device("cuda")
    weights = wan_model.WanWeights(CFG, device, seed=4)
    model = wan_model.WanTransformer(weights, GRID, wan_model.SequenceShard(),
                                     wan_model.fused_prologue(CFG.heads, CFG.eps))
    g = torch.Generator(device=device)
    g.manual_seed(5)
    latent = torch.randn((CFG.in_channels, GRID[0], 2 * GRID[1], 2 * GRID[2]), generator=g,
                         device=device)
    text = [torch.randn((1, CFG.text_tokens, CFG.text_dim), generator=g, device=device,
                        dtype=torch.bfloat16) for _ in range(2)]
    contexts = {b: model.context(text[b]) for b in (0, 1)}
    reset_runtime_state()

    def attention(q, k, v):
        return parallel.head_parallel_attention(q, k, v, lambda a, b, c: backend(a, b, c),
                                                None, 1)
    out = wan_model.denoise(model, wan_model.patchify(latent, CFG), contexts, attention,
                            wan_model.CfgCombine(5.0), steps=STEPS)
    torch.cuda.synchronize()
    _native.check_device_errors()
    return out


def test_full_routes_match_dense_generation():
    dense = generate(DenseBackend())
    flex = FlexReuseBackend(FlexReuseConfig(bootstrap_mode="sampled", route_samples=16,
                                            sampled_update_interval=2,
                                            prefetch_sampled_update=False, keep=1.0,
                                            mass_target=1.0, spatial_reorder=True,
                                            total_steps=STEPS))
    sparse = generate(flex)
    assert torch.isfinite(sparse).all()
    # layer 1 of both branches ran the sparse kernels at steps 1 and 2
    assert flex.phase_counts["sparse_reuse"] == 2 * 2
    assert flex.phase_counts["first_layer_dense"] == 2 * STEPS
    err = (sparse - dense).abs()
    scale = dense.abs().mean()
    assert err.max() <= 0.05 * dense.abs().max(), (err.max(), dense.abs().max())
    assert err.mean() <= 0.02 * scale, (err.mean(), scale)


def test_recommended_flags_phases():
    flex = FlexReuseBackend(FlexReuseConfig(bootstrap_mode="sampled", route_samples=16,
                                            sampled_update_interval=2,
                                            prefetch_sampled_update=False, keep=0.625,
                                            mass_target=0.95, dense_route_threshold=0.58,
                                            spatial_reorder=True, total_steps=STEPS))
    out = generate(flex)
    assert torch.isfinite(out).all()
    counts = flex.phase_counts
    assert counts["first_layer_dense"] == 2 * STEPS
    assert counts["sampled_bootstrap"] == 2                 # layer 1, both branches, step 0
    # steps 1 and 2 of layer 1 either reuse the route or were dispatched dense
    assert counts["sparse_reuse"] + counts["dense_dispatch"] == 2 * 2
    assert flex.profile_summary()["released_routes"] == 2   # released at the final step
