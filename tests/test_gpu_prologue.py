"""GPU parity of the attention prologue (``csrc/prologue.cu``: RMSNorm of Q/K,
RoPE, reorder in one pass) through the C ABI, against the reference's
outputs (``tests/golden/prologue.npz``) and the oracle: bit-exact."""

import numpy as np
import pytest
import torch

from dit_sparse_atten_b200 import _native, kernels, synthetic
from dit_sparse_atten_b200.spatial import build_spatial_layout
from oracle import prologue as opro
from test_oracle_prologue import CASE, bf16_bits_to_float, prologue_case

pytestmark = pytest.mark.gpu
DEV = "cuda"


def run(proj, weights, rotary, heads, perm, eps=1e-6, norm=(True, True), rope=True):
    qp, kp, vp = (x.to(DEV) for x in proj)
    wq, wk = weights
    cos = rotary.real.float() if rope else None
    sin = rotary.imag.float() if rope else None
    out = kernels.qkv_prologue(qp, kp, vp, heads, wq, wk, eps, cos, sin,
                               perm=None if perm is None else torch.as_tensor(perm),
                               norm_q=norm[0], norm_k=norm[1])
    torch.cuda.synchronize()
    _native.check_device_errors()
    return [o.float().cpu().numpy() for o in out]


def oracle(proj, weights, rotary, heads, perm, eps=1e-6, norm=(True, True), rope=True):
    qp, kp, vp = (x.float().cpu().numpy() for x in proj)
    wq, wk = (None if w is None else w.float().numpy() for w in weights)
    return opro.qkv_prologue(qp, kp, vp, heads, wq if norm[0] else False,
                             wk if norm[1] else False, eps,
                             rotary.real.numpy() if rope else None,
                             rotary.imag.numpy() if rope else None, perm=perm)


def test_matches_reference_fixture(golden):
    g = golden("prologue.npz")
    proj, weights, rotary = prologue_case()
    got = run(proj, weights, rotary, CASE["heads"], g["perm"])
    for name, arr in zip("qkv", got):
        assert np.array_equal(arr, bf16_bits_to_float(g[name])), name


@pytest.mark.parametrize("batch,grid,heads,variant", [
    (2, (2, 5, 48), 40, "full"),       # Wan heads, 480 tokens, partial last block
    (1, (2, 8, 16), 3, "no_weight"),
    (1, (2, 8, 16), 3, "no_rope"),
    (2, (1, 8, 16), 2, "no_norm_k"),
    (1, (2, 8, 16), 2, "strided"),     # projections as column slices of one [B, T, 3C] tensor
])
def test_matches_oracle(batch, grid, heads, variant):
    proj, weights, rotary = synthetic.prologue_inputs(batch, grid, heads, seed=heads + batch)
    perm = build_spatial_layout(grid, 128).permutation_cpu.numpy()
    kw = {}
    if variant == "no_weight":
        weights = (None, None)
    if variant == "no_rope":
        kw["rope"] = False
    if variant == "no_norm_k":
        kw["norm"] = (True, False)
    if variant == "strided":
        fused = torch.cat(proj, -1)
        C = proj[0].shape[-1]
        proj = [fused[..., i * C:(i + 1) * C] for i in range(3)]
        assert proj[0].stride(1) == 3 * C
    got = run(proj, weights, rotary, heads, perm, **kw)
    ref = oracle(proj, weights, rotary, heads, perm, **kw)
    for name, a, r in zip("qkv", got, ref):
        assert np.array_equal(a, r), (name, int((a != r).sum()))


def test_identity_order_and_bad_perm_entry():
    proj, weights, rotary = synthetic.prologue_inputs(1, (1, 8, 16), 2, seed=3)
    got = run(proj, weights, rotary, 2, None)
    ref = oracle(proj, weights, rotary, 2, None)
    assert all(np.array_equal(a, r) for a, r in zip(got, ref))
    perm = torch.arange(128, dtype=torch.int32)
    perm[5] = 500
    kernels.qkv_prologue(*(x.to(DEV) for x in proj), 2, *weights, 1e-6, rotary.real.float(),
                         rotary.imag.float(), perm=perm)
    with pytest.raises(RuntimeError, match="out of range"):
        _native.check_device_errors()


class _Norm:
    def __init__(self, weight, eps=1e-6):
        self.weight, self.eps = weight, eps


class _WanAttention(torch.nn.Module):
    """The attributes of diffusers' WanAttention that the processor uses."""

    def __init__(self, heads, head_dim, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        dim = heads * head_dim
        self.heads = heads

        def linear():
            lin = torch.nn.Linear(dim, dim, bias=True)
            with torch.no_grad():
                lin.weight.copy_(torch.randn((dim, dim), generator=g) * dim ** -0.5)
                lin.bias.copy_(torch.randn(dim, generator=g) * 0.1)
            return lin.to(DEV, torch.bfloat16)
        self.to_q, self.to_k, self.to_v = linear(), linear(), linear()
        self.to_out = torch.nn.ModuleList([linear(), torch.nn.Identity()])
        self.norm_q = _Norm((torch.rand(dim, generator=g) + 0.5).to(DEV, torch.bfloat16))
        self.norm_k = _Norm((torch.rand(dim, generator=g) + 0.5).to(DEV, torch.bfloat16))


def test_processor_matches_backend_on_unpacked_inputs(monkeypatch):
    """The processor's packed hand-over gives bit for bit the output of the same
    backend fed unpacked, prologue-normalised inputs, through a bootstrap step
    and a sparse reuse step; the first (dense) layer keeps the original order."""
    from dit_sparse_atten_b200 import flex as flex_module
    from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig
    from dit_sparse_atten_b200.processor import StudyWanProcessor
    from dit_sparse_atten_b200.prologue import rope_tables

    grid, heads = (4, 16, 32), 2
    attn = _WanAttention(heads, 128, seed=4)
    _, _, rotary = synthetic.prologue_inputs(1, grid, heads, seed=5)
    rot = rotary[None, None].to(DEV)
    g = torch.Generator().manual_seed(6)
    hidden = torch.randn((1, 2048, heads * 128), generator=g).to(DEV, torch.bfloat16)
    cfg = FlexReuseConfig(spatial_reorder=True, keep=0.5, mass_target=0.9)
    fused_backend, plain_backend = FlexReuseBackend(cfg), FlexReuseBackend(cfg)
    processor = StudyWanProcessor(fused_backend, layer_id=1)
    cos, sin = rope_tables(rot)
    for step in (0, 1):
        monkeypatch.setattr(flex_module, "routing_context",
                            lambda include_grid=False, s=step: (1, s, 0, grid) if include_grid
                            else (1, s, 0))
        got = processor(attn, hidden, rotary_emb=rot)
        q, k, v = kernels.qkv_prologue(attn.to_q(hidden), attn.to_k(hidden), attn.to_v(hidden),
                                       heads, attn.norm_q.weight, attn.norm_k.weight, 1e-6,
                                       cos, sin)
        ref = plain_backend(q, k, v, dtype=q.dtype).flatten(2, 3)
        ref = attn.to_out[0](ref)
        torch.cuda.synchronize()
        _native.check_device_errors()
        assert torch.equal(got, ref), step
    assert fused_backend.phase_counts["sparse_reuse"] == 1
    # layer 0 is dense in the backend: the processor's inputs must not be packed
    monkeypatch.setattr(flex_module, "routing_context",
                        lambda include_grid=False: (0, 0, 0, grid) if include_grid else (0, 0, 0))
    layer0 = StudyWanProcessor(FlexReuseBackend(cfg), layer_id=0)
    assert layer0.backend.packed_layout_for(2048) is None
    out0 = layer0(attn, hidden, rotary_emb=rot)
    q, k, v = kernels.qkv_prologue(attn.to_q(hidden), attn.to_k(hidden), attn.to_v(hidden),
                                   heads, attn.norm_q.weight, attn.norm_k.weight, 1e-6, cos, sin)
    dense = torch.nn.functional.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
    torch.testing.assert_close(out0, attn.to_out[0](dense.flatten(2, 3)), atol=2e-2, rtol=2e-2)
