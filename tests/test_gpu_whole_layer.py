"""Whole-layer parity of the block-sparse attention at full size.

Every (branch, head, query block) row of config 4 (2 x 40 x 450 = 36,000 rows,
57,600 tokens, Morton-packed) and of config 2 (2 x 12 x 256 = 6,144 rows,
32,760 tokens, partial last block of 120 tokens) is checked against an fp32
reference, and so is the full-size output of ``FlexReuseBackend.__call__`` with
the spatial reorder and the unpack folded into the attention's store (the
bench's end-to-end API).

The fp32 reference is ``oracle/attention.py``'s block-sparse attention restated
with torch on the GPU so that a whole layer fits in seconds: for each (branch,
head) and chunk of query blocks, scores against all keys in float32 (TF32
off), keys of unrouted blocks and keys past the last token masked out,
softmax, PV; rows with an empty route are zero.  It is pinned to the numpy
oracle on a subset of rows in the same test.  Semantics: the reference's
``sparse_chunk`` (``attention_backends/sparse.py:670-751``).

Bars: max-abs 2e-2 and mean-abs 2e-3 over all rows.
"""

import math

import numpy as np
import pytest
import torch

from conftest import unpack_route
from dit_sparse_atten_b200 import _native, kernels, synthetic
from dit_sparse_atten_b200.context import reset_runtime_state, set_routing_context
from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig
from dit_sparse_atten_b200.spatial import build_spatial_layout
from oracle import attention as oatt

pytestmark = pytest.mark.gpu

DEV = "cuda"
MAX_ABS = 2e-2
MEAN_ABS = 2e-3
PIN_ATOL = 1e-4          # torch fp32 reference vs numpy fp32 oracle (summation order only)


@torch.no_grad()
def fp32_reference(q, k, v, route, block, chunk=16):
    """fp32 block-sparse attention of bf16 ``q, k, v [B, T, H, D]`` over a bool
    route ``[B, H, Qb, Kb]`` (or ``[H, Qb, Kb]`` shared by the batch); returns
    fp32 ``[B, T, H, D]`` on the GPU."""
    B, T, H, D = q.shape
    blocks = math.ceil(T / block)
    route = torch.as_tensor(route, device=q.device)
    if route.dim() == 3:
        route = route.unsqueeze(0).expand(B, -1, -1, -1)
    out = torch.empty((B, T, H, D), dtype=torch.float32, device=q.device)
    scale = D ** -0.5
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for b in range(B):
            for h in range(H):
                qf, kf, vf = (x[b, :, h].float() for x in (q, k, v))
                for qb0 in range(0, blocks, chunk):
                    qb1 = min(blocks, qb0 + chunk)
                    r0, r1 = qb0 * block, min(T, qb1 * block)
                    s = (qf[r0:r1] @ kf.T) * scale
                    keep = route[b, h, qb0:qb1].repeat_interleave(block, 0)[: r1 - r0]
                    keep = keep.repeat_interleave(block, 1)[:, :T]
                    s.masked_fill_(~keep, float("-inf"))
                    p = torch.softmax(s, -1).nan_to_num_(0.0)   # empty routes -> zero rows
                    out[b, r0:r1, h] = p @ vf
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    return out


def assert_all_rows_close(actual, expected):
    """max-abs and mean-abs over every element, reduced on the GPU."""
    diff = (actual.float() - expected).abs()
    assert torch.isfinite(diff).all()
    max_abs, mean_abs = float(diff.max()), float(diff.mean())
    assert max_abs <= MAX_ABS, max_abs
    assert mean_abs <= MEAN_ABS, mean_abs
    return max_abs, mean_abs


def pin_to_oracle(ref, q, k, v, route, block, b, heads, qbs):
    """The torch fp32 reference equals the numpy oracle on these rows."""
    route = np.asarray(route)
    r = route[b] if route.ndim == 4 else route
    qs, ks, vs = (x[b][:, heads].float().cpu().numpy() for x in (q, k, v))
    expect = oatt.block_sparse_attention(qs, ks, vs, r[heads], block, query_blocks=qbs,
                                         dtype=np.float32)
    T = q.shape[1]
    rows = np.concatenate([np.arange(qb * block, min(T, qb * block + block)) for qb in qbs])
    got = ref[b][:, heads].cpu().numpy()
    np.testing.assert_allclose(got[rows], expect[rows], atol=PIN_ATOL, rtol=0)


@pytest.fixture(scope="module")
def config4(golden):
    cfg = synthetic.CONFIG4
    routes = unpack_route(golden("blob_routes.npz")["c4_route"], cfg.blocks)   # packed order
    lay = build_spatial_layout(cfg.grid, 128)
    q, k, v = synthetic.wan_qkv(cfg, seed=41, device=DEV)
    qp, kp, vp = lay.reorder_qkv(q, k, v)
    ref_p = fp32_reference(qp, kp, vp, routes, 128)
    return cfg, routes, lay, (q, k, v), (qp, kp, vp), ref_p


def test_config4_every_row(config4):
    cfg, routes, _lay, _raw, (qp, kp, vp), ref_p = config4
    pin_to_oracle(ref_p, qp, kp, vp, routes, 128, b=1, heads=[0, 21, 39], qbs=[0, 224, 449])
    counts, indices = kernels.pack_boolean_rows(torch.from_numpy(routes).to(DEV))
    out_p = kernels.block_sparse_attention(qp, kp, vp, counts, indices, block=128)
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert out_p.shape == ref_p.shape
    assert_all_rows_close(out_p, ref_p)


def test_config4_backend_api_every_row(config4):
    """FlexReuseBackend.__call__ per CFG branch, reuse phase, spatial reorder on:
    raster in, raster out (the unpack folded into the attention's store)."""
    cfg, routes, lay, (q, k, v), _packed, ref_p = config4
    ref = lay.restore(ref_p)                       # fp32 reference in raster order
    backend = FlexReuseBackend(FlexReuseConfig(spatial_reorder=True, bootstrap_mode="sampled",
                                               keep=cfg.keep, mass_target=cfg.mass_target))
    reset_runtime_state()
    try:
        for b in range(cfg.batch):
            backend.install_route(torch.from_numpy(routes[b]), attention_id=1, branch=b,
                                  tokens=cfg.tokens, heads=cfg.heads, head_dim=cfg.head_dim,
                                  device=q.device, grid=cfg.grid)
        for b in range(cfg.batch):
            set_routing_context(attention_id=1, step=1, branch=b, grid=cfg.grid)
            out = backend(q[b:b + 1], k[b:b + 1], v[b:b + 1])
            torch.cuda.synchronize()
            _native.check_device_errors()
            assert out.shape == (1, cfg.tokens, cfg.heads, cfg.head_dim)
            assert out.dtype == torch.bfloat16
            assert_all_rows_close(out[0], ref[b])
        assert backend.phase_counts["sparse_reuse"] == cfg.batch
    finally:
        reset_runtime_state()


def test_config2_every_row(golden):
    """Config 2 (480p, raster order, partial last block of 120 tokens)."""
    cfg = synthetic.CONFIG2
    routes = unpack_route(golden("blob_routes.npz")["c2_route"], cfg.blocks)
    q, k, v = synthetic.wan_qkv(cfg, seed=21, device=DEV)
    ref = fp32_reference(q, k, v, routes, 128)
    pin_to_oracle(ref, q, k, v, routes, 128, b=0, heads=[0, 11],
                  qbs=[0, 128, cfg.blocks - 1])
    counts, indices = kernels.pack_boolean_rows(torch.from_numpy(routes).to(DEV))
    out = kernels.block_sparse_attention(q, k, v, counts, indices, block=128)
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert cfg.tokens % 128 == 120
    assert_all_rows_close(out, ref)
