"""Freeze golden fixtures from the reference study itself.

Run in a container where the reference checkout is mounted; it is imported
from the directory named by ``$BSA_REFERENCE``, which must be set::

    BSA_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Inputs are regenerated in the tests from the seeded generators of
``dit_sparse_atten_b200.synthetic`` and checked against the SHA-256 digests
stored here, so only reference *outputs* (and small inputs) are committed.
Fixtures:

* ``kat.json``        the reference tests' own known answers
                      (tests/test_flex_backend.py:16-27,56-59;
                      tests/test_flex_route_update.py:106-112;
                      tests/test_spatial_layout.py:6-29) re-run through the
                      reference functions.
* ``layouts.npz``     ``build_spatial_layout`` outputs for four grids and the
                      sparse backend's tile-major permutation for config 1.
* ``config1.npz``     config 1 through the reference sparse backend's
                      ``sparse_chunk`` (tile-major, tile 64).
* ``route_480p.npz``  ``_sampled_block_mass`` (S=16 and S=2) on a 2-head 480p
                      case with a partial tail block, the persistence prior,
                      ``_top_mass_route`` and the sink; exact block mass
                      (``_reference_block_mass``) with a partial tail.
* ``config3.npz``     the full config-3 route decision (57,600 tokens, 40 heads):
                      digests of Q/K, reference mass of two heads, the
                      reference route and counts.
* ``blob_routes.npz`` config-2 and config-4 routes from the seeded blob scores.
* ``prologue.npz``    the Wan processor's Q/K ``rms_norm`` and ``apply_rope``
                      (``svg_ops.py:82-92,193-204`` CPU path) on seeded
                      projections, reordered by the reference's layout.
* ``directional.npz`` ``directional_budget_update`` (``routing.py:97-168``) and
                      the sunk route / frontier of ``_add_first_frame_sink``
                      on the config-3 mass of two heads (plain, and quantised
                      so that equal scores straddle the budget cut), three
                      option sets each.
"""

from __future__ import annotations

import hashlib
import json
import math
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
if not os.environ.get("BSA_REFERENCE"):
    raise SystemExit("set BSA_REFERENCE to the reference checkout (the directory that holds "
                     "attention_backends/)")
sys.path.insert(0, os.environ["BSA_REFERENCE"])

from attention_backends import flex as ref_flex  # noqa: E402
from attention_backends import layout_ops as ref_layout_ops  # noqa: E402
from attention_backends import routing as ref_routing  # noqa: E402
from attention_backends import svg_ops as ref_svg_ops  # noqa: E402
from attention_backends import sparse as ref_sparse  # noqa: E402
from attention_backends import spatial as ref_spatial  # noqa: E402

from dit_sparse_atten_b200 import synthetic  # noqa: E402


def sha256(t: torch.Tensor) -> str:
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def packbits(route: torch.Tensor) -> np.ndarray:
    return np.packbits(route.numpy().astype(bool), axis=-1)


def kat():
    out = {}
    mass = torch.tensor([[[0.50, 0.30, 0.15, 0.05]]])
    out["top_mass"] = {"mass": mass.tolist(), "target": 0.90, "keep": 0.50,
                       "route": ref_flex._top_mass_route(mass, 0.90, 0.50).tolist()}
    route = torch.tensor([[[True, False, True], [False, True, False]],
                          [[False, True, True], [True, False, True]]])
    counts, indices = ref_flex._pack_route(route)
    out["pack"] = {"route": route.tolist(), "counts": counts.tolist(), "indices": indices.tolist()}
    backend = ref_flex.FlexReuseBackend(ref_flex.FlexReuseConfig(block_size=128))
    sunk = backend._add_first_frame_sink({"grid": (2, 8, 16), "layout": None},
                                         {"route": torch.zeros(2, 4, 4, dtype=torch.bool)})
    out["sink"] = {"grid": [2, 8, 16], "shape": [2, 4, 4], "route": sunk["route"].tolist()}
    lay = ref_spatial.build_spatial_layout((16, 45, 80), block_size=128)
    out["layout_720p"] = {"microtile": list(lay.microtile_shape), "tokens": lay.tokens,
                          "blocks": lay.blocks}
    lay = ref_spatial.build_spatial_layout((2, 4, 8), block_size=8, max_microtile_tokens=8)
    out["layout_small"] = {"microtile": list(lay.microtile_shape)}
    # sampled(S=block) == exact / block, reference test_flex_backend.py:43-53
    torch.manual_seed(4)
    q = torch.randn(1, 12, 2, 8)
    k = torch.randn_like(q)
    scores = torch.einsum("bqhd,bkhd->bhqk", q, k) * 8 ** -0.5
    exact = ref_flex._block_attention_mass(q, k, scores.logsumexp(-1), 4)
    sampled = ref_flex._sampled_block_mass(q, k, 4, samples=4)
    out["sampled_full"] = {"q": q.tolist(), "k": k.tolist(), "exact": exact.tolist(),
                           "sampled": sampled.tolist()}
    (HERE / "kat.json").write_text(json.dumps(out))


def layouts():
    arrays = {}
    for name, grid, block, mt in (("720p", (16, 45, 80), 128, 32), ("480p", (21, 30, 52), 128, 32),
                                  ("small", (2, 4, 8), 8, 8), ("c1", (3, 8, 16), 64, 32)):
        lay = ref_spatial.build_spatial_layout(grid, block, mt)
        arrays[f"{name}_microtile"] = np.array(lay.microtile_shape)
        arrays[f"{name}_perm"] = lay.permutation_cpu.numpy()
        arrays[f"{name}_inverse"] = lay.inverse_cpu.numpy()
        arrays[f"{name}_neighbors"] = lay.neighbors_cpu.numpy()
        arrays[f"{name}_block_frames"] = lay.block_frames_cpu.numpy()
    tl = ref_sparse._spatial_layout((3, 8, 16), 64, 384)
    arrays["c1_tile"] = np.array([tl.tile_h, tl.tile_w])
    idx = torch.arange(384).reshape(1, 384, 1, 1).float()
    arrays["c1_tile_major"] = tl.to_tile_major(idx).reshape(-1).long().numpy().astype(np.int32)
    np.savez_compressed(HERE / "layouts.npz", **arrays)


def config1():
    q, k, v, route = synthetic.config1_inputs(seed=0)
    tl = ref_sparse._spatial_layout((3, 8, 16), 64, 384)
    qt, kt, vt = (tl.to_tile_major(x) for x in (q, k, v))
    tiles = 384 // 64
    stats = ref_sparse._empty_route_stats(12, tiles, "cpu")
    out_t = ref_sparse.sparse_chunk(qt, kt, vt, route, 64, 0, 384, None, stats)
    out = tl.from_tile_major(out_t)
    # dense masked softmax in raster order, for the record
    perm = tl.to_tile_major(torch.arange(384).reshape(1, 384, 1, 1).float()).reshape(-1).long()
    tile_of = torch.empty(384, dtype=torch.long)
    tile_of[perm] = torch.arange(384) // 64
    allowed = route[:, tile_of[:, None], tile_of[None, :]]
    qh, kh, vh = (x[0].permute(1, 0, 2) for x in (q, k, v))
    dense = ((qh @ kh.transpose(-1, -2)) * 128 ** -0.5).masked_fill(~allowed, -torch.inf)
    dense = (dense.softmax(-1) @ vh).permute(1, 0, 2).unsqueeze(0)
    np.savez_compressed(
        HERE / "config1.npz",
        q_sha=sha256(q), k_sha=sha256(k), v_sha=sha256(v), route=route.numpy(),
        output=out.numpy(), dense_masked_maxabs=np.float32((out - dense).abs().max()))


def route_480p():
    cfg = synthetic.LayerConfig("route480p", (21, 30, 52), 1, 2, 128)
    q, k = synthetic.structured_qk(cfg, seed=7)
    arrays = {"q_sha": sha256(q), "k_sha": sha256(k)}
    for s in (16, 2):
        arrays[f"mass_s{s}"] = ref_flex._sampled_block_mass(q, k, 128, samples=s).numpy()
    mass = torch.from_numpy(arrays["mass_s16"])
    prev = synthetic.previous_route(2, 256, seed=70)
    prior = mass + 0.5 * mass.mean(-1, keepdim=True) * prev.float()
    route = ref_flex._top_mass_route(prior, 0.95, 0.625)
    backend = ref_flex.FlexReuseBackend(ref_flex.FlexReuseConfig(block_size=128))
    sunk = backend._add_first_frame_sink({"grid": (21, 30, 52), "layout": None},
                                         {"route": route})["route"]
    counts, indices = ref_layout_ops.pack_boolean_rows(sunk)
    arrays.update(prev=packbits(prev), prior=prior.numpy(), route_nosink=packbits(route),
                  route=packbits(sunk), counts=counts.numpy(), indices=indices.numpy().astype(np.int16),
                  keep=np.float32(sunk.float().mean()))
    # exact mass with a partial tail block (reference tests/test_flex_backend.py:62-75 shape)
    torch.manual_seed(2)
    qe = torch.randn(1, 259, 3, 16)
    ke = torch.randn_like(qe)
    lse = (torch.einsum("bqhd,bkhd->bhqk", qe, ke) * 16 ** -0.5).logsumexp(-1)
    arrays.update(exact_q=qe.numpy(), exact_k=ke.numpy(),
                  exact_mass=ref_flex._block_attention_mass(qe, ke, lse, block_size=128).numpy())
    np.savez_compressed(HERE / "route_480p.npz", **arrays)


def config3():
    cfg = synthetic.CONFIG3
    t0 = time.time()
    q, k = synthetic.structured_qk(cfg, seed=3)
    prev = synthetic.previous_route(cfg.heads, cfg.blocks, seed=33)
    mass = ref_flex._sampled_block_mass(q, k, 128, samples=16)
    prior = mass + 0.5 * mass.mean(-1, keepdim=True) * prev.float()
    route = ref_flex._top_mass_route(prior, 0.95, 0.625)
    backend = ref_flex.FlexReuseBackend(ref_flex.FlexReuseConfig(block_size=128))
    sunk = backend._add_first_frame_sink({"grid": cfg.grid, "layout": None},
                                         {"route": route})["route"]
    counts, _ = ref_layout_ops.pack_boolean_rows(sunk)
    heads = np.array([0, 17])
    np.savez_compressed(
        HERE / "config3.npz", q_sha=sha256(q), k_sha=sha256(k), prev=packbits(prev),
        heads=heads, mass_heads=mass[heads].numpy(), route=packbits(sunk),
        counts=counts.numpy().astype(np.int16),
        kept_per_head=sunk.reshape(cfg.heads, -1).sum(-1).numpy(),
        keep=np.float32(sunk.float().mean()), seconds=np.float32(time.time() - t0))


def blob_routes():
    arrays = {}
    for name, cfg in (("c2", synthetic.CONFIG2), ("c4", synthetic.CONFIG4)):
        routes = []
        for branch in range(cfg.batch):
            scores = synthetic.blob_scores(cfg.heads, cfg.blocks, seed=100 + branch)
            arrays[f"{name}_scores_sha{branch}"] = sha256(scores)
            route = ref_flex._top_mass_route(scores, cfg.mass_target, cfg.keep)
            route[..., :cfg.sink_blocks] = True
            routes.append(packbits(route))
        arrays[f"{name}_route"] = np.stack(routes)
    np.savez_compressed(HERE / "blob_routes.npz", **arrays)


DIRECTIONAL_OPTIONS = (
    {},
    {"min_ratio": 0.5, "candidate_bonus": 0.25, "budget_scale": 1.1,
     "exploration_fraction": 0.02, "expand_joint": False},
    {"persistence": 0.0, "expand_k": False, "expand_joint": False, "budget_scale": 0.9,
     "exploration_fraction": 0.5},
)


def directional_inputs(c3):
    """Masses and previous route of the directional fixtures (the tests rebuild
    them the same way and check the digests)."""
    heads = c3["heads"]
    mass = torch.from_numpy(c3["mass_heads"])
    prev = torch.from_numpy(np.unpackbits(c3["prev"], axis=-1, count=450).astype(bool))[heads]
    quant = torch.round(mass * (450 * 64.0)) / (450 * 64.0)
    return {"plain": mass, "quant": quant}, prev


def directional():
    c3 = np.load(HERE / "config3.npz")
    masses, prev = directional_inputs(c3)
    lay = ref_spatial.build_spatial_layout((16, 45, 80), block_size=128)
    nb = lay.neighbors_cpu
    backend = ref_flex.FlexReuseBackend(ref_flex.FlexReuseConfig(block_size=128))
    arrays = {}
    for mname, mass in masses.items():
        arrays[f"{mname}_sha"] = sha256(mass)
        for i, opts in enumerate(DIRECTIONAL_OPTIONS):
            result = ref_routing.directional_budget_update(
                mass, prev, nb, keep=0.625, previous_frontier=ref_routing.frontier_mask(prev, nb),
                **opts)
            for key, value in result.items():
                arrays[f"{mname}{i}_{key}"] = packbits(value)
            sunk = backend._add_first_frame_sink({"grid": (16, 45, 80), "layout": lay}, result)
            arrays[f"{mname}{i}_sunk_route"] = packbits(sunk["route"])
            arrays[f"{mname}{i}_sunk_frontier"] = packbits(sunk["frontier"])
    arrays["options"] = np.array(json.dumps(DIRECTIONAL_OPTIONS))
    np.savez_compressed(HERE / "directional.npz", **arrays)


PROLOGUE_CASE = {"batch": 1, "grid": (1, 8, 16), "heads": 2, "seed": 12, "eps": 1e-6}


def prologue():
    c = PROLOGUE_CASE
    (qp, kp, vp), (wq, wk), rotary = synthetic.prologue_inputs(c["batch"], c["grid"], c["heads"],
                                                               seed=c["seed"])
    lay = ref_spatial.build_spatial_layout(c["grid"], block_size=128)
    heads = c["heads"]

    def run(x, w):
        x = ref_svg_ops.rms_norm(x.contiguous(), w, c["eps"])
        return x.unflatten(2, (heads, -1)).transpose(1, 2).contiguous()
    q, k = run(qp, wq), run(kp, wk)
    q, k = ref_svg_ops.apply_rope(q, k, rotary[None, None])
    v = vp.unflatten(2, (heads, -1))
    q, k = q.transpose(1, 2), k.transpose(1, 2)
    q, k, v = lay.reorder_qkv(q.contiguous(), k.contiguous(), v.contiguous())
    np.savez_compressed(
        HERE / "prologue.npz", proj_sha=np.array([sha256(x) for x in (qp, kp, vp)]),
        weight_sha=np.array([sha256(w) for w in (wq, wk)]), rotary_sha=sha256(torch.view_as_real(rotary)),
        perm=lay.permutation_cpu.numpy(), q=q.contiguous().view(torch.int16).numpy(),
        k=k.contiguous().view(torch.int16).numpy(), v=v.contiguous().view(torch.int16).numpy())


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    only = set(sys.argv[1:])
    for fn in (kat, layouts, config1, route_480p, blob_routes, config3, directional, prologue):
        if only and fn.__name__ not in only:
            continue
        t = time.time()
        fn()
        print(f"{fn.__name__}: {time.time() - t:.1f}s")


if __name__ == "__main__":
    main()
