"""GPU parity of the block-sparse attention kernel (a).

Tolerance: bf16 output within max-abs 2e-2 and
mean-abs 2e-3 of the fp32 reference.
"""

import math

import numpy as np
import pytest
import torch

from conftest import unpack_route
from dit_sparse_atten_b200 import _native, kernels, synthetic
from dit_sparse_atten_b200.spatial import build_spatial_layout, tile_major_layout
from oracle import attention as oatt
from oracle import route as oroute

pytestmark = pytest.mark.gpu

DEV = "cuda"
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def assert_attention_close(actual, expected, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    diff = np.abs(np.asarray(actual, np.float64) - np.asarray(expected, np.float64))
    assert np.isfinite(diff).all()
    assert diff.max() <= max_abs, diff.max()
    assert diff.mean() <= mean_abs, diff.mean()


def run(q, k, v, route, block, **kw):
    """Attention through the CSR built on the GPU; route bool [H, Qb, Kb] or [B, H, Qb, Kb]."""
    counts, indices = kernels.pack_boolean_rows(torch.as_tensor(route, device=DEV))
    out = kernels.block_sparse_attention(q.to(DEV), k.to(DEV), v.to(DEV), counts, indices,
                                         block=block, **kw)
    torch.cuda.synchronize()
    _native.check_device_errors()
    return out


def test_config1_block64_matches_reference(golden):
    g = golden("config1.npz")
    q, k, v, route = synthetic.config1_inputs(seed=0)
    lay = tile_major_layout((3, 8, 16), 8, 8)
    qb, kb, vb = (x.to(torch.bfloat16).to(DEV) for x in (q, k, v))
    qt, kt, vt = lay.reorder_qkv(qb, kb, vb)
    out_t = run(qt, kt, vt, route, 64)
    out = lay.restore(out_t).float().cpu().numpy()
    assert_attention_close(out, g["output"])


@pytest.mark.parametrize("tokens,heads,block,density,seed", [
    (256, 2, 128, 0.6, 0), (250, 2, 128, 0.5, 1), (1000, 3, 128, 0.3, 2),
    (777, 2, 64, 0.5, 3), (384, 4, 64, 0.8, 4), (4096, 2, 128, 0.625, 5)])
def test_random_routes_match_oracle(tokens, heads, block, density, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn((1, tokens, heads, 128), generator=g).to(torch.bfloat16)
               for _ in range(3))
    blocks = math.ceil(tokens / block)
    route = torch.rand((heads, blocks, blocks), generator=g) < density
    route |= torch.eye(blocks, dtype=torch.bool)
    out = run(q, k, v, route, block)
    ref = oatt.block_sparse_attention(q[0].float().numpy(), k[0].float().numpy(),
                                      v[0].float().numpy(), route.numpy(), block)
    assert_attention_close(out[0].float().cpu().numpy(), ref)


def test_reference_explicit_block_mask_case():
    """tests/test_flex_backend.py:122-148 at head_dim 128: identity route, partial tail."""
    torch.manual_seed(1)
    q, k, v = (torch.randn(1, 250, 2, 128).to(torch.bfloat16) for _ in range(3))
    route = torch.eye(2, dtype=torch.bool).expand(2, -1, -1).contiguous()
    out = run(q, k, v, route, 128)
    ref = oatt.dense_masked_attention(q[0].float().numpy(), k[0].float().numpy(),
                                      v[0].float().numpy(), route.numpy(), 128)
    assert_attention_close(out[0].float().cpu().numpy(), ref)


def test_empty_rows_are_zero_and_lse():
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn((2, 300, 2, 128), generator=g).to(torch.bfloat16) for _ in range(3))
    route = torch.rand((2, 2, 3, 3), generator=g) < 0.5
    route[0, 0, 1] = False
    route[1, 1, 2] = True
    counts, indices = kernels.pack_boolean_rows(route.to(DEV))
    out, lse = kernels.block_sparse_attention(q.to(DEV), k.to(DEV), v.to(DEV), counts, indices,
                                              block=128, return_lse=True)
    torch.cuda.synchronize()
    for b in range(2):
        ref, ref_lse = oatt.block_sparse_attention(
            q[b].float().numpy(), k[b].float().numpy(), v[b].float().numpy(),
            route[b].numpy(), 128, return_lse=True)
        got = out[b].float().cpu().numpy()
        assert_attention_close(got, ref)
        lse_got = lse[b].cpu().numpy()
        finite = np.isfinite(ref_lse)
        np.testing.assert_allclose(lse_got[finite], ref_lse[finite], atol=2e-2, rtol=1e-3)
        assert np.isneginf(lse_got[~finite]).all()
    assert (out[0, 128:256, 0] == 0).all()


def test_many_items_per_cta_with_empty_rows():
    """More (b, h, qb) work items than CTAs resident on the GPU at once (later
    CTAs start as earlier ones retire), empty routes among them, a partial tail."""
    g = torch.Generator().manual_seed(9)
    B, H, T = 2, 4, 128 * 100 - 5
    blocks = math.ceil(T / 128)
    q, k, v = (torch.randn((B, T, H, 128), generator=g).to(torch.bfloat16) for _ in range(3))
    route = torch.rand((B, H, blocks, blocks), generator=g) < 0.08
    route[..., 0] = True
    empty = torch.rand((B, H, blocks), generator=g) < 0.1
    route[empty] = False
    counts, indices = kernels.pack_boolean_rows(route.to(DEV))
    out, lse = kernels.block_sparse_attention(q.to(DEV), k.to(DEV), v.to(DEV), counts, indices,
                                              block=128, return_lse=True)
    torch.cuda.synchronize()
    _native.check_device_errors()
    for b in range(B):
        ref, ref_lse = oatt.block_sparse_attention(
            q[b].float().numpy(), k[b].float().numpy(), v[b].float().numpy(),
            route[b].numpy(), 128, return_lse=True)
        assert_attention_close(out[b].float().cpu().numpy(), ref)
        lse_got = lse[b].cpu().numpy()
        finite = np.isfinite(ref_lse)
        np.testing.assert_allclose(lse_got[finite], ref_lse[finite], atol=2e-2, rtol=1e-3)
        assert np.isneginf(lse_got[~finite]).all()
    assert empty.any()


def test_shared_route_across_batch():
    g = torch.Generator().manual_seed(8)
    q, k, v = (torch.randn((2, 512, 2, 128), generator=g).to(torch.bfloat16) for _ in range(3))
    route = torch.rand((2, 4, 4), generator=g) < 0.6
    route |= torch.eye(4, dtype=torch.bool)
    out = run(q, k, v, route, 128)
    for b in range(2):
        ref = oatt.block_sparse_attention(q[b].float().numpy(), k[b].float().numpy(),
                                          v[b].float().numpy(), route.numpy(), 128)
        assert_attention_close(out[b].float().cpu().numpy(), ref)


def test_config2_480p_layer(golden):
    """Full config 2 (B=2, 32,760 tokens, 12 heads, partial tail) on blob routes."""
    cfg = synthetic.CONFIG2
    routes = unpack_route(golden("blob_routes.npz")["c2_route"], cfg.blocks)
    q, k, v = synthetic.wan_qkv(cfg, seed=21, device=DEV)
    out = run(q, k, v, torch.from_numpy(routes), 128)
    assert torch.isfinite(out).all()
    heads = [0, 5, 11]
    qbs = [0, 1, 100, cfg.blocks - 2, cfg.blocks - 1]
    rows = np.concatenate([np.arange(qb * 128, min(cfg.tokens, qb * 128 + 128)) for qb in qbs])
    for b in range(cfg.batch):
        qs, ks, vs = (x[b][:, heads].float().cpu().numpy() for x in (q, k, v))
        ref = oatt.block_sparse_attention(qs, ks, vs, routes[b][heads], 128, query_blocks=qbs,
                                          dtype=np.float32)
        got = out[b][:, heads].float().cpu().numpy()
        assert_attention_close(got[rows], ref[rows])


def test_config4_720p_layer_morton(golden):
    """Config 4 (B=2, 57,600 tokens, 40 heads): pack, attention, unpack; sampled rows."""
    cfg = synthetic.CONFIG4
    routes = unpack_route(golden("blob_routes.npz")["c4_route"], cfg.blocks)
    lay = build_spatial_layout(cfg.grid, 128)
    q, k, v = synthetic.wan_qkv(cfg, seed=41, device=DEV)
    qp, kp, vp = lay.reorder_qkv(q, k, v)
    out_p = run(qp, kp, vp, torch.from_numpy(routes), 128)
    out = lay.restore(out_p)
    torch.cuda.synchronize()
    assert torch.isfinite(out_p).all()
    heads = [0, 13, 39]
    qbs = [0, 7, 225, 449]
    rows = np.concatenate([np.arange(qb * 128, qb * 128 + 128) for qb in qbs])
    for b in range(cfg.batch):
        qs, ks, vs = (x[b][:, heads].float().cpu().numpy() for x in (qp, kp, vp))
        ref = oatt.block_sparse_attention(qs, ks, vs, routes[b][heads], 128, query_blocks=qbs,
                                          dtype=np.float32)
        got = out_p[b][:, heads].float().cpu().numpy()
        assert_attention_close(got[rows], ref[rows])
    perm = lay.permutation_cpu.long().to(DEV)
    assert torch.equal(out[:, perm[:512]].view(torch.int16), out_p[:, :512].view(torch.int16))


def test_exp2_paths_accuracy():
    """Both softmax exponentials against float64 and CUDA's exp2f (torch.exp2),
    evaluated by the test-only diagnostic library."""
    import diag

    x = torch.cat([torch.linspace(-126.0, 8.0, 1 << 20), torch.tensor([0.0, -0.5, 0.5, 7.99])])
    ref = np.exp2(x.double().numpy())
    xd = x.to(DEV)
    poly = diag.exp2(xd, "poly").double().cpu().numpy()
    mufu = diag.exp2(xd, "mufu").double().cpu().numpy()
    cuda_exp2f = torch.exp2(xd).double().cpu().numpy()
    normal = x.numpy() >= -125.0            # results >= 2^-125 stay normal floats
    assert (np.abs(poly - ref) / ref)[normal].max() <= 1e-4
    assert np.abs(poly - ref)[~normal].max() <= 2.0 ** -125 * 1e-3
    assert (np.abs(mufu - ref) / ref)[normal].max() <= 2.0 ** -21
    assert (np.abs(poly - cuda_exp2f) / cuda_exp2f)[normal].max() <= 1e-4 + 2.0 ** -22
    below = diag.exp2(torch.tensor([-200.0, -1000.0], device=DEV), "poly").cpu()
    assert (below >= 0).all() and (below < 2.0 ** -125).all()


@pytest.mark.parametrize("grid,block,batch,heads", [((2, 16, 32), 128, 2, 3),
                                                    ((3, 8, 16), 64, 1, 2),
                                                    ((5, 30, 52), 128, 2, 2)])
def test_scatter_store_equals_attention_then_restore(grid, block, batch, heads):
    """The unpack folded into the output store (bsa_attention_fwd_scatter) is
    bit-identical to attention in packed order followed by the layout's
    restore, partial last blocks (5x30x52 = 7,800 tokens) and batch included."""
    lay = build_spatial_layout(grid, block)
    tokens = grid[0] * grid[1] * grid[2]
    blocks = math.ceil(tokens / block)
    g = torch.Generator().manual_seed(tokens + heads)
    q, k, v = (torch.randn((batch, tokens, heads, 128), generator=g).to(torch.bfloat16).to(DEV)
               for _ in range(3))
    route = torch.rand((heads, blocks, blocks), generator=g) < 0.55
    route[:, :, 0] = True
    counts, indices = kernels.pack_boolean_rows(route.to(DEV))
    qp, kp, vp = lay.reorder_qkv(q, k, v)
    ref = lay.restore(kernels.block_sparse_attention(qp, kp, vp, counts, indices, block=block))
    perm = lay.permutation_cpu.to(DEV)
    got, lse = kernels.block_sparse_attention(qp, kp, vp, counts, indices, block=block,
                                              out_rows=perm, return_lse=True)
    _, lse_ref = kernels.block_sparse_attention(qp, kp, vp, counts, indices, block=block,
                                                return_lse=True)
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(lse, lse_ref)           # the LSE stays in packed row order


def test_scatter_store_reports_out_of_range_rows():
    tokens, heads = 256, 1
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn((1, tokens, heads, 128), generator=g).to(torch.bfloat16).to(DEV)
               for _ in range(3))
    route = torch.ones((heads, 2, 2), dtype=torch.bool)
    counts, indices = kernels.pack_boolean_rows(route.to(DEV))
    rows = torch.arange(tokens, dtype=torch.int32)
    rows[7] = tokens + 5                       # no row is written to token 7
    out = torch.zeros_like(q)
    kernels.block_sparse_attention(q, k, v, counts, indices, out=out, out_rows=rows.to(DEV))
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="out of range"):
        _native.check_device_errors()
    assert out[0, 7].abs().sum().item() == 0
    assert out[0, 8].abs().sum().item() > 0
