"""GPU parity of the route decision (b) and the reorder (c) against the oracle / reference."""

import math

import numpy as np
import pytest
import torch

from conftest import sha256_tensor, unpack_route
from dit_sparse_atten_b200 import _native, kernels, synthetic
from oracle import layout as olay
from oracle import route as oroute

pytestmark = pytest.mark.gpu

DEV = "cuda"


def assert_mass_close(actual, expected):
    """Mass tolerance; see tests/test_oracle_golden.py::assert_mass_close."""
    diff = np.abs(np.asarray(actual, np.float64) - np.asarray(expected, np.float64))
    assert diff.max() <= 2e-3, diff.max()
    assert diff.mean() <= 2e-6, diff.mean()
    close = diff <= 2e-4 * np.abs(np.asarray(expected, np.float64)) + 1e-7
    assert close.mean() >= 0.995, close.mean()


def select(mass, prev=None, persistence=0.0, target=0.95, keep=0.625, sink=0):
    r = kernels.route_select(torch.as_tensor(mass, device=DEV),
                             None if prev is None else torch.as_tensor(prev, device=DEV),
                             persistence, target, keep, sink)
    torch.cuda.synchronize()
    return r


def check_csr(result, route):
    counts, indices = oroute.pack_boolean_rows(route)
    np.testing.assert_array_equal(result.route.cpu().numpy().astype(bool), route)
    np.testing.assert_array_equal(result.counts.cpu().numpy(), counts)
    np.testing.assert_array_equal(result.indices.cpu().numpy(), indices)


# ----------------------------------------------------------------------------
# (c) reorder
# ----------------------------------------------------------------------------

@pytest.mark.parametrize("shape,dtype", [((2, 64, 3, 17), torch.bfloat16),
                                          ((1, 1000, 2, 128), torch.bfloat16),
                                          ((3, 333, 5), torch.float32),
                                          ((2, 77, 3), torch.uint8)])
def test_reorder_matches_index_select(shape, dtype):
    g = torch.Generator().manual_seed(1)
    xs = [(torch.randn(shape, generator=g) * 100).to(dtype) for _ in range(3)]
    perm = torch.randperm(shape[1], generator=g).to(torch.int32)
    out = kernels.reorder_rows([x.to(DEV) for x in xs], perm.to(DEV))
    for o, x in zip(out, xs):
        np.testing.assert_array_equal(o.cpu().view(torch.uint8).numpy(),
                                      olay.reorder(x.view(torch.uint8).numpy(), perm.numpy()))


def test_reorder_morton_round_trip_config4_size():
    from dit_sparse_atten_b200.spatial import build_spatial_layout
    cfg = synthetic.CONFIG4
    lay = build_spatial_layout(cfg.grid, 128)
    g = torch.Generator(device=DEV).manual_seed(2)
    q, k, v = (torch.randn((cfg.batch, cfg.tokens, cfg.heads, 128), generator=g, device=DEV,
                           dtype=torch.bfloat16) for _ in range(3))
    qp, kp, vp = lay.reorder_qkv(q, k, v)
    back = lay.restore(kp)
    torch.cuda.synchronize()
    assert torch.equal(back.view(torch.int16), k.view(torch.int16))
    idx = torch.randint(0, cfg.tokens, (64,))
    perm = lay.permutation_cpu.long()
    for t in idx.tolist():
        assert torch.equal(qp[:, t].view(torch.int16), q[:, perm[t]].view(torch.int16))
        assert torch.equal(vp[:, t].view(torch.int16), v[:, perm[t]].view(torch.int16))
    _native.check_device_errors()


def test_reorder_flags_out_of_range_permutation():
    x = torch.zeros((1, 8, 16), device=DEV, dtype=torch.bfloat16)
    perm = torch.tensor([0, 1, 2, 3, 4, 5, 6, 99], dtype=torch.int32, device=DEV)
    kernels.reorder_rows([x], perm)
    with pytest.raises(RuntimeError, match="out of range"):
        _native.check_device_errors()


# ----------------------------------------------------------------------------
# CSR pack
# ----------------------------------------------------------------------------

def test_pack_matches_stable_reference():
    torch.manual_seed(19)  # reference tests/test_flex_backend.py:30-40
    route = torch.rand(5, 37, 450) < 0.61
    counts, indices = kernels.pack_boolean_rows(route.to(DEV))
    ec, ei = oroute.pack_boolean_rows(route.numpy())
    np.testing.assert_array_equal(counts.cpu().numpy(), ec)
    np.testing.assert_array_equal(indices.cpu().numpy(), ei)


def test_pack_kat(golden):
    k = golden("kat.json")["pack"]
    counts, indices = kernels.pack_boolean_rows(torch.tensor(k["route"], device=DEV))
    assert counts[None].tolist() == k["counts"]
    assert indices[None].tolist() == k["indices"]


# ----------------------------------------------------------------------------
# (b) selection: bit-exact from the same fp32 mass
# ----------------------------------------------------------------------------

def test_top_mass_kat(golden):
    k = golden("kat.json")["top_mass"]
    r = select(np.array(k["mass"], np.float32), target=k["target"], keep=k["keep"])
    assert r.route.bool().tolist() == k["route"]


def test_select_480p_fixture_bit_exact(golden):
    g = golden("route_480p.npz")
    prev = unpack_route(g["prev"], 256)
    r = select(g["mass_s16"], prev, 0.5, 0.95, 0.625, sink=13)
    route = unpack_route(g["route"], 256)
    check_csr(r, route)
    np.testing.assert_array_equal(r.indices.cpu().numpy(), g["indices"])
    assert r.kept.cpu().tolist() == route.reshape(2, -1).sum(-1).tolist()
    # without sink / prior
    r = select(g["prior"], target=0.95, keep=0.625)
    np.testing.assert_array_equal(r.route.cpu().numpy().astype(bool),
                                  unpack_route(g["route_nosink"], 256))


def test_select_config3_fixture_heads_bit_exact(golden):
    g = golden("config3.npz")
    cfg = synthetic.CONFIG3
    heads = g["heads"]
    prev = unpack_route(g["prev"], cfg.blocks)[heads]
    r = select(g["mass_heads"], prev, 0.5, 0.95, 0.625, sink=cfg.sink_blocks)
    check_csr(r, unpack_route(g["route"], cfg.blocks)[heads])


@pytest.mark.parametrize("name,cfg", [("c2", synthetic.CONFIG2), ("c4", synthetic.CONFIG4)])
def test_select_blob_routes_bit_exact(golden, name, cfg):
    g = golden("blob_routes.npz")
    routes = unpack_route(g[f"{name}_route"], cfg.blocks)
    for branch in range(cfg.batch):
        scores = synthetic.blob_scores(cfg.heads, cfg.blocks, seed=100 + branch)
        assert sha256_tensor(scores) == str(g[f"{name}_scores_sha{branch}"])
        r = kernels.route_select(scores.to(DEV), target=cfg.mass_target, keep=cfg.keep,
                                 sink_blocks=cfg.sink_blocks)
        torch.cuda.synchronize()
        check_csr(r, routes[branch])


@pytest.mark.parametrize("cols", [5, 17, 256, 450, 1000])
def test_select_tie_heavy_rows_match_oracle(cols):
    rng = np.random.default_rng(cols)
    for levels in (2, 4, 9):
        mass = (rng.integers(1, levels + 1, (64, cols)) / levels).astype(np.float32)
        prev = rng.random((64, cols)) < 0.5
        r = select(mass, prev, 0.5, 0.9, 0.625, sink=1)
        ref = oroute.sampled_route(mass, prev, 0.5, 0.9, 0.625)
        ref[..., :1] = True
        assert oroute.boundary_ties(oroute.persistence_prior(mass, prev, 0.5), 0.9, 0.625).any()
        check_csr(r, ref)


def _row_families(rng, rows, cols):
    """Rows that take each branch of the selection kernels: wide-range masses
    (the parallel float64 prefix sums are exact), masses spanning ~70 decades
    (not provably exact: serial scan), zeros, negative values (non-monotone
    prefix sums), and exactly tied values."""
    u = rng.random((rows, cols))
    wide = u ** 4
    decades = np.exp(-rng.random((rows, cols)) * 160.0)
    zeros = np.where(rng.random((rows, cols)) < 0.4, 0.0, u)
    signed = rng.standard_normal((rows, cols))
    tied = rng.integers(0, 3, (rows, cols)) / 2.0
    return [x.astype(np.float32) for x in (wide, decades, zeros, signed, tied)]


@pytest.mark.parametrize("cols", [1, 2, 7, 31, 32, 33, 64, 65, 128, 129, 255, 256, 300, 450,
                                  511, 512, 513])
def test_select_row_families_every_width(cols):
    """Every register width of the warp kernel (and the CTA kernel above 512
    blocks) against the oracle, with and without the prior, caps from 1 to
    all blocks."""
    rng = np.random.default_rng(1000 + cols)
    for mass in _row_families(rng, 24, cols):
        prev = rng.random(mass.shape) < 0.5
        for target, keep in ((0.95, 0.625), (1.0, 1.0), (0.5, 1e-9), (0.999, 0.9)):
            r = select(mass, target=target, keep=keep)
            check_csr(r, oroute.top_mass_route(mass, target, keep))
            r = select(mass, prev, 0.5, target, keep, sink=min(cols, 3))
            ref = oroute.sampled_route(mass, prev, 0.5, target, keep)
            ref[..., :3] = True
            check_csr(r, ref)
            kept = r.kept.cpu().numpy()
            assert kept.tolist() == ref.reshape(len(kept), -1).sum(-1).tolist()


def test_select_random_keep_and_target_sweep():
    rng = np.random.default_rng(3)
    mass = (rng.random((8, 40, 450)) ** 4).astype(np.float32)
    for target, keep in ((0.5, 0.3), (0.9, 0.625), (0.99, 1.0), (1.0, 0.58)):
        r = select(mass, target=target, keep=keep)
        check_csr(r, oroute.top_mass_route(mass, target, keep))


# ----------------------------------------------------------------------------
# (b) sampled and exact mass
# ----------------------------------------------------------------------------

def test_sampled_mass_480p_matches_reference(golden):
    g = golden("route_480p.npz")
    cfg = synthetic.LayerConfig("route480p", (21, 30, 52), 1, 2, 128)
    q, k = synthetic.structured_qk(cfg, seed=7)
    assert sha256_tensor(q) == str(g["q_sha"])
    for s in (16, 2):
        mass = kernels.sampled_block_mass(q.to(DEV), k.to(DEV), 128, s)
        torch.cuda.synchronize()
        assert_mass_close(mass[0].cpu().numpy(), g[f"mass_s{s}"])
    _native.check_device_errors()


@pytest.mark.parametrize("T,block,samples", [(1000, 128, 1), (3000, 128, 2), (4096, 64, 4),
                                             (2500, 128, 8), (57600, 128, 16), (1900, 64, 32),
                                             (61000, 128, 16), (5000, 128, 32)])
def test_sampled_mass_one_pass_matches_two_pass(T, block, samples):
    """One pass over the sampled keys against the two-pass kernel, partial
    last blocks included; rows sum to 1.  16 or 32 samples and at most 473
    blocks keep the per-row block log-sums on chip (no workspace: 57,600 and
    5,000 tokens); other shapes go through a workspace and a reduction
    launch (61,000 tokens: 477 blocks).
    Both kernels take a quarter of their exponentials from a polynomial with
    relative error <= 7.5e-5, evaluated at different arguments (running vs
    final stabiliser), hence rtol 2e-4 (the mass parity bound)."""
    g = torch.Generator().manual_seed(T + samples)
    q, k = (torch.randn((2, T, 3, 128), generator=g).to(torch.bfloat16).to(DEV)
            for _ in range(2))
    one = kernels.sampled_block_mass(q, k, block, samples)
    two = kernels.sampled_block_mass(q, k, block, samples, one_pass=False)
    torch.cuda.synchronize()
    _native.check_device_errors()
    torch.testing.assert_close(one, two, atol=1e-6, rtol=2e-4)
    rows = one.double().sum(-1)
    torch.testing.assert_close(rows, torch.ones_like(rows), atol=1e-4, rtol=0)


def test_route_decision_config3(golden):
    """Full config 3: mass vs reference, bit-exact selection from the GPU mass."""
    g = golden("config3.npz")
    cfg = synthetic.CONFIG3
    q, k = synthetic.structured_qk(cfg, seed=3)
    assert sha256_tensor(q) == str(g["q_sha"]) and sha256_tensor(k) == str(g["k_sha"])
    prev = unpack_route(g["prev"], cfg.blocks)
    mass = kernels.sampled_block_mass(q.to(DEV), k.to(DEV), 128, 16)[0]
    r = kernels.route_select(mass, torch.from_numpy(prev).to(DEV), 0.5, 0.95, 0.625,
                             cfg.sink_blocks)
    torch.cuda.synchronize()
    _native.check_device_errors()
    m = mass.cpu().numpy()
    assert_mass_close(m[g["heads"]], g["mass_heads"])
    ref = oroute.sampled_route(m, prev, 0.5, 0.95, 0.625, grid=cfg.grid, block=128)
    check_csr(r, ref)
    agreement = (r.route.cpu().numpy().astype(bool) == unpack_route(g["route"], cfg.blocks)).mean()
    assert agreement >= 0.995, agreement
    keep = oroute.route_keep(ref)
    assert abs(keep - float(g["keep"])) < 0.01


def test_exact_mass_partial_tail_matches_oracle():
    g = torch.Generator().manual_seed(5)
    q = torch.randn((1, 259, 3, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((1, 259, 3, 128), generator=g).to(torch.bfloat16)
    mass = kernels.exact_block_mass(q.to(DEV), k.to(DEV), 128)
    torch.cuda.synchronize()
    qf, kf = q[0].double().numpy(), k[0].double().numpy()
    scores = np.einsum("qhd,khd->hqk", qf, kf) * 128 ** -0.5
    mx = scores.max(-1, keepdims=True)
    lse = (mx + np.log(np.exp(scores - mx).sum(-1, keepdims=True)))[..., 0]
    ref = oroute.exact_block_mass(qf, kf, lse, 128)
    np.testing.assert_allclose(mass[0].cpu().numpy(), ref, atol=2e-3, rtol=1e-3)
    np.testing.assert_allclose(mass[0].sum(-1).cpu().numpy(),
                               np.array([[128, 128, 3]] * 3, np.float32), rtol=1e-3)


def test_sampled_full_equals_exact_over_block():
    """Reference identity sampled(S=block) == exact / block (tests/test_flex_backend.py:43-53)."""
    g = torch.Generator().manual_seed(4)
    q = torch.randn((1, 512, 2, 128), generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn((1, 512, 2, 128), generator=g).to(torch.bfloat16).to(DEV)
    exact = kernels.exact_block_mass(q, k, 32)
    sampled = kernels.sampled_block_mass(q, k, 32, 32, round_bf16=False)
    torch.cuda.synchronize()
    np.testing.assert_allclose(sampled.cpu().numpy(), exact.cpu().numpy() / 32, rtol=1e-4,
                               atol=1e-7)
    np.testing.assert_allclose(exact.sum(-1).cpu().numpy(), 32.0, rtol=1e-3)


def _exact_reference(q, k, block):
    """float64 oracle mass and LSE of bf16 ``q, k [1, T, H, D]``."""
    qf, kf = q[0].double().cpu().numpy(), k[0].double().cpu().numpy()
    scores = np.einsum("qhd,khd->hqk", qf, kf) * 128 ** -0.5
    mx = scores.max(-1, keepdims=True)
    lse = (mx + np.log(np.exp(scores - mx).sum(-1, keepdims=True)))[..., 0]
    return oroute.exact_block_mass(qf, kf, lse, block), lse


@pytest.mark.parametrize("tokens,heads,block", [
    (5000, 2, 128),     # 40 key tiles: three groups of the cross-warp reduction, partial tail
    (1000, 3, 64),      # 64-token blocks: two query and two key blocks per tile
    (4096, 1, 128),     # exactly two full groups
])
def test_exact_mass_wide_blocks_match_oracle_and_repeat(tokens, heads, block):
    g = torch.Generator().manual_seed(tokens + heads)
    q = torch.randn((1, tokens, heads, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((1, tokens, heads, 128), generator=g).to(torch.bfloat16)
    ref, lse = _exact_reference(q, k, block)
    qd, kd = q.to(DEV), k.to(DEV)
    first = kernels.exact_block_mass(qd, kd, block)
    second = kernels.exact_block_mass(qd, kd, block)
    given = kernels.exact_block_mass(qd, kd, block,
                                     lse=torch.from_numpy(lse).float().unsqueeze(0).to(DEV))
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert torch.equal(first, second)                       # deterministic reduction order
    np.testing.assert_allclose(first[0].cpu().numpy(), ref, atol=2e-3, rtol=1e-3)
    np.testing.assert_allclose(given[0].cpu().numpy(), ref, atol=2e-3, rtol=1e-3)
    torch.testing.assert_close(given, first, atol=1e-4, rtol=1e-4)
    rows = np.minimum(block, tokens - np.arange(ref.shape[1]) * block)
    np.testing.assert_allclose(first[0].sum(-1).cpu().numpy(),
                               np.broadcast_to(rows, ref.shape[:2]), rtol=1e-3)


def test_exact_mass_from_attention_lse_batch2():
    """The bootstrap's pairing: LSE of the routed attention over a full route,
    then one mass pass; batch 2 with a partial tail."""
    g = torch.Generator().manual_seed(3)
    B, T, H = 2, 1500, 2
    q, k, v = (torch.randn((B, T, H, 128), generator=g).to(torch.bfloat16).to(DEV)
               for _ in range(3))
    blocks = math.ceil(T / 128)
    full = torch.ones((B, H, blocks, blocks), dtype=torch.bool, device=DEV)
    counts, indices = kernels.pack_boolean_rows(full)
    _, lse = kernels.block_sparse_attention(q, k, v, counts, indices, 128, return_lse=True)
    mass = kernels.exact_block_mass(q, k, 128, lse=lse)
    two_pass = kernels.exact_block_mass(q, k, 128)
    torch.cuda.synchronize()
    _native.check_device_errors()
    torch.testing.assert_close(mass, two_pass, atol=1e-4, rtol=1e-3)
    for b in range(B):
        ref, _ = _exact_reference(q[b:b + 1].cpu(), k[b:b + 1].cpu(), 128)
        np.testing.assert_allclose(mass[b].cpu().numpy(), ref, atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("B,T,H,workspace", [(2, 1500, 3, 2 << 30), (1, 2200, 4, 1)])
def test_dense_attention_block_mass(B, T, H, workspace):
    """One dense pass gives the output and LSE of the all-blocks routed
    attention (bit for bit) and the exact block mass; a tiny workspace forces
    one head per launch."""
    g = torch.Generator().manual_seed(T + H)
    q, k, v = (torch.randn((B, T, H, 128), generator=g).to(torch.bfloat16).to(DEV)
               for _ in range(3))
    out, lse, mass = kernels.dense_attention_block_mass(q, k, v, workspace_bytes=workspace)
    blocks = math.ceil(T / 128)
    full = torch.ones((B, H, blocks, blocks), dtype=torch.bool, device=DEV)
    counts, indices = kernels.pack_boolean_rows(full)
    ref_out, ref_lse = kernels.block_sparse_attention(q, k, v, counts, indices, 128,
                                                      return_lse=True)
    two_pass = kernels.exact_block_mass(q, k, 128)
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
    assert torch.equal(lse, ref_lse)
    torch.testing.assert_close(mass, two_pass, atol=2e-5, rtol=1e-4)
    for b in range(B):
        ref, _ = _exact_reference(q[b:b + 1].cpu(), k[b:b + 1].cpu(), 128)
        np.testing.assert_allclose(mass[b].cpu().numpy(), ref, atol=2e-3, rtol=1e-3)


def test_gather_scatter_rows_with_offsets():
    """bsa_gather_scatter_rows: src/dst row maps, three tensors into one
    buffer at row offsets, out-of-range map entries skipped and reported."""
    g = torch.Generator().manual_seed(4)
    src = [torch.randn((1, 50, 2, 8), generator=g).to(DEV) for _ in range(3)]
    src_rows = torch.randint(0, 50, (30,), generator=g, dtype=torch.int32)
    dst_rows = torch.randperm(40, generator=g)[:30].to(torch.int32)
    buf = torch.zeros((1, 120, 2, 8), device=DEV)
    kernels.gather_scatter_rows(src, [buf] * 3, src_rows.to(DEV), dst_rows.to(DEV),
                                dst_offsets=[0, 40, 80])
    torch.cuda.synchronize()
    _native.check_device_errors()
    expect = torch.zeros_like(buf)
    for t in range(3):
        expect[0, 40 * t + dst_rows.long()] = src[t][0, src_rows.long()]
    assert torch.equal(buf, expect)
    bad = dst_rows.clone()
    bad[3] = 500
    kernels.gather_scatter_rows(src[:1], [buf], src_rows.to(DEV), bad.to(DEV))
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="out of range"):
        _native.check_device_errors()
