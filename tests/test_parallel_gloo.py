"""Head-parallel (Ulysses) exchange and the keep all-reduce on 2 CPU ranks (gloo)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dit_sparse_atten_b200 import parallel


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        queue.put((rank, fn(rank, world)))
    except Exception as exc:  # reported to the parent
        queue.put((rank, exc))
    finally:
        dist.destroy_process_group()


def run_ranks(fn, world=2):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, value in results.items():
        if isinstance(value, Exception):
            raise value
    return results


def full_inputs():
    g = torch.Generator().manual_seed(0)
    return [torch.randn((1, 64, 4, 8), generator=g) for _ in range(3)]


def _exchange(rank, world):
    q, _, _ = full_inputs()
    t = q.shape[1] // world
    shard = q[:, rank * t:(rank + 1) * t]
    heads = parallel.seq_to_head(shard, dist.group.WORLD, world)
    hp = q.shape[2] // world
    assert torch.equal(heads, q[:, :, rank * hp:(rank + 1) * hp])
    back = parallel.head_to_seq(heads, dist.group.WORLD, world)
    assert torch.equal(back, shard)
    return True


class CpuRows:
    """The exchange's row moves with torch indexing (the product uses the
    CUDA row-gather kernels): the host-side layout logic under test."""

    @staticmethod
    def gather(tensors, perm):
        return tuple(t.index_select(1, perm.long()) for t in tensors)

    @staticmethod
    def scatter(srcs, dsts, src_rows, dst_rows, dst_offsets=None):
        offsets = dst_offsets or [0] * len(dsts)
        for src, dst, off in zip(srcs, dsts, offsets):
            dst[:, off + dst_rows.long()] = src[:, src_rows.long()]


def _attention(rank, world):
    q, k, v = full_inputs()
    t = q.shape[1] // world
    sl = slice(rank * t, (rank + 1) * t)

    def attend(qh, kh, vh):
        return torch.nn.functional.scaled_dot_product_attention(
            qh.transpose(1, 2), kh.transpose(1, 2), vh.transpose(1, 2)).transpose(1, 2)

    out = parallel.head_parallel_attention(q[:, sl], k[:, sl], v[:, sl], attend,
                                           dist.group.WORLD, world, rows=CpuRows)
    ref = attend(q, k, v)[:, sl]
    torch.testing.assert_close(out, ref)
    # batch 2 takes the generic (concatenating) exchange
    q2, k2, v2 = (torch.cat([x, x.flip(1)], 0) for x in (q, k, v))
    out2 = parallel.head_parallel_attention(q2[:, sl], k2[:, sl], v2[:, sl], attend,
                                            dist.group.WORLD, world)
    torch.testing.assert_close(out2, attend(q2, k2, v2)[:, sl])
    return True


def _pipelined(rank, world):
    q, k, v = full_inputs()
    t = q.shape[1] // world
    sl = slice(rank * t, (rank + 1) * t)
    perm = torch.randperm(q.shape[1], generator=torch.Generator().manual_seed(3))
    inverse = torch.empty_like(perm)
    inverse[perm] = torch.arange(perm.numel())
    seen = []

    def sdpa(qh, kh, vh):
        return torch.nn.functional.scaled_dot_product_attention(
            qh.transpose(1, 2), kh.transpose(1, 2), vh.transpose(1, 2)).transpose(1, 2)

    def attend(qp, kp, vp, chunk, out, out_rows):
        seen.append(chunk)
        return sdpa(qp, kp, vp)         # permutation-equivariant: output stays in pack order

    def attend_scatter(qp, kp, vp, chunk, out, out_rows):
        # the folded unpack: write row i to token out_rows[i]
        res = sdpa(qp, kp, vp)
        rows = torch.arange(res.shape[1]) if out_rows is None else out_rows.long()
        out[:, rows] = res
        return None

    ref = sdpa(q, k, v)[:, sl]
    for kw in ({"perm": perm, "inverse": inverse, "chunks": 2}, {"chunks": 1}, {"chunks": 2}):
        for fn in (attend, attend_scatter):
            seen.clear()
            pipe = parallel.PipelinedHeadParallel(dist.group.WORLD, world, q.shape[2], t,
                                                  rows=CpuRows, **kw)
            out = pipe(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(), fn)
            torch.testing.assert_close(out, ref)
            if fn is attend:
                assert seen == list(range(kw["chunks"]))
    # the packed inputs of a chunk are exactly this rank's heads in pack order
    got = {}

    def capture(qp, kp, vp, chunk, out, out_rows):
        got[chunk] = qp.clone()
        return qp
    pipe = parallel.PipelinedHeadParallel(dist.group.WORLD, world, q.shape[2], t, perm=perm,
                                          inverse=inverse, chunks=2, rows=CpuRows)
    pipe(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(), capture)
    hp = q.shape[2] // world
    for c in range(2):
        head = rank * hp + c
        assert torch.equal(got[c][0, :, 0], q[0, perm, head])
    return True


def cpu_block_sparse_attention(q, k, v, counts, indices, block=128, scale=None, out=None,
                               return_lse=False, out_rows=None):
    """fp32 CPU stand-in for ``kernels.block_sparse_attention`` (same
    arguments and output placement) for the host-side tests."""
    B, T, H, D = q.shape
    scale = scale or D ** -0.5
    res = torch.empty_like(q)
    for h in range(H):
        for qb in range(counts.shape[-1]):
            n = int(counts[h, qb])
            keys = torch.cat([torch.arange(kb * block, min((kb + 1) * block, T))
                              for kb in indices[h, qb, :n].tolist()])
            rows = torch.arange(qb * block, min((qb + 1) * block, T))
            s = q[0, rows, h].float() @ k[0, keys, h].float().T * scale
            res[0, rows, h] = (torch.softmax(s, -1) @ v[0, keys, h].float()).to(q.dtype)
    dst = out if out is not None else torch.empty_like(q)
    if out_rows is not None:
        dst[:, out_rows.long()] = res
    else:
        dst.copy_(res)
    return dst


def cpu_pack_boolean_rows(route):
    counts = route.sum(-1).to(torch.int32)
    order = torch.argsort((~route).to(torch.int8), dim=-1, stable=True)
    return counts, order.to(torch.int32)


def _backend_head_parallel(rank, world):
    """FlexReuseBackend.head_parallel on a reuse call: the chunked, overlapped
    exchange gives the same output as all heads through __call__ and as the
    unsharded routed attention; other calls take the unchunked exchange."""
    from dit_sparse_atten_b200 import flex, kernels
    from dit_sparse_atten_b200.context import set_routing_context
    from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig

    kernels.block_sparse_attention = cpu_block_sparse_attention
    kernels.pack_boolean_rows = cpu_pack_boolean_rows
    kernels.reorder_rows = lambda tensors, perm: tuple(x.index_select(1, perm.long())
                                                       for x in tensors)
    flex.frontier_mask = lambda route, neighbors: None
    grid, heads, d = (2, 16, 16), 4, 16
    tokens = 512
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn((1, tokens, heads, d), generator=g).to(torch.bfloat16)
               for _ in range(3))
    route = torch.rand((heads, 4, 4), generator=g) < 0.6
    route[:, torch.arange(4), torch.arange(4)] = True
    t = tokens // world
    sl = slice(rank * t, (rank + 1) * t)
    hp = heads // world
    backend = FlexReuseBackend(FlexReuseConfig(spatial_reorder=True))
    backend.install_route(route[rank * hp:(rank + 1) * hp], attention_id=1, branch=0,
                          tokens=tokens, heads=hp, head_dim=d, device=torch.device("cpu"),
                          grid=grid)
    set_routing_context(attention_id=1, step=1, branch=0, grid=grid)
    shard = [x[:, sl].contiguous() for x in (q, k, v)]
    piped = backend.head_parallel(*shard, dist.group.WORLD, world, rows=CpuRows, chunks=2)
    assert backend.pipelines, "reuse call must take the chunked exchange"
    assert backend.phase_counts["sparse_reuse"] == 1
    plain = backend.head_parallel(*shard, dist.group.WORLD, world, rows=CpuRows,
                                  deterministic=True)    # not the pipelined form
    assert backend.phase_counts["sparse_reuse"] == 2 and len(backend.pipelines) == 1
    # unsharded: pack, routed attention over all heads, unpack
    layout = backend._spatial_layout(grid, tokens)
    perm = layout.permutation_cpu.long()
    counts, indices = cpu_pack_boolean_rows(route)
    ref = cpu_block_sparse_attention(q[:, perm], k[:, perm], v[:, perm], counts, indices,
                                     out_rows=perm)
    torch.testing.assert_close(piped, ref[:, sl], atol=2e-2, rtol=0)
    torch.testing.assert_close(plain, piped, atol=2e-2, rtol=0)
    return True


def _peer_fallback(rank, world):
    """Peer exchange set-up failing on one rank: every rank learns it from the
    group (a MIN all-reduce), and the pipelined call takes the all-to-all
    exchange with equal chunks instead, output unchanged.  The CUDA IPC calls
    are replaced by host fakes; no device memory is mapped."""
    from dit_sparse_atten_b200 import kernels

    def export(t):
        if rank == 1:
            raise RuntimeError("cannot export this allocation")
        return bytes(range(64)), 256
    kernels.ipc_export = export
    kernels.ipc_import = lambda handle, device: 1 << 20
    shards = parallel.PeerShards(dist.group.WORLD, world, (4, 2, 8), torch.float32, "cpu")
    assert not shards.ready
    assert (shards.error is not None) == (rank == 1)
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn((1, 32, 10, 8), generator=g) for _ in range(3))
    t = q.shape[1] // world
    sl = slice(rank * t, (rank + 1) * t)
    perm = torch.randperm(q.shape[1], generator=torch.Generator().manual_seed(6))
    inverse = torch.empty_like(perm)
    inverse[perm] = torch.arange(perm.numel())

    def attend(qp, kp, vp, chunk, out, out_rows, peers=None):
        assert peers is None, "no peer stores after a failed set-up"
        return torch.nn.functional.scaled_dot_product_attention(
            qp.transpose(1, 2), kp.transpose(1, 2), vp.transpose(1, 2)).transpose(1, 2)

    pipe = parallel.PipelinedHeadParallel(dist.group.WORLD, world, 10, t, perm=perm,
                                          inverse=inverse, chunks=5, rows=CpuRows,
                                          peer_out=True, peer_in=True)
    assert [(s.start, s.stop) for s in pipe.chunk_slices()] == [(0, 1), (1, 5)]
    out = pipe(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(), attend)
    ref = attend(q, k, v, 0, None, None)[:, sl]
    torch.testing.assert_close(out, ref)
    assert not pipe.peer_in and not pipe.peer_out
    assert (pipe.peer_error is not None) == (rank == 1)
    assert [(s.start, s.stop) for s in pipe.chunk_slices()] == [(c, c + 1) for c in range(5)]
    # every rank exports: the shards are mapped, this rank's own by address
    kernels.ipc_export = lambda t: (bytes(range(64)), 256)
    shards = parallel.PeerShards(dist.group.WORLD, world, (4, 2, 8), torch.float32, "cpu")
    assert shards.ready and shards.error is None
    assert shards.ptrs[rank] == shards.local.data_ptr()
    assert shards.ptrs[1 - rank] == (1 << 20) + 256
    return True


def _keep(rank, world):
    from dit_sparse_atten_b200.flex import FlexReuseBackend
    backend = FlexReuseBackend(process_group=dist.group.WORLD)
    kept = torch.tensor([3, 5]) if rank == 0 else torch.tensor([7, 1])
    return backend._global_keep(kept, 2 * 4 * 4)


def test_seq_head_exchange_round_trip():
    assert all(run_ranks(_exchange).values())


def test_head_parallel_attention_equals_full():
    assert all(run_ranks(_attention).values())


def test_pipelined_exchange_equals_full_attention():
    assert all(run_ranks(_pipelined).values())


def test_backend_head_parallel_pipelines_reuse_calls():
    assert all(run_ranks(_backend_head_parallel).values())


def test_peer_exchange_falls_back_on_every_rank():
    assert all(run_ranks(_peer_fallback).values())


def test_pipeline_chunk_rule():
    assert [parallel.pipeline_chunks(h) for h in (40, 20, 10, 5, 8, 12, 3)] == [4, 4, 2, 1, 2, 2, 1]
    with pytest.raises(ValueError):
        parallel.PipelinedHeadParallel(None, 2, 40, 16, chunks=3)
    with pytest.raises(ValueError):
        parallel.PipelinedHeadParallel(None, 2, 40, 16, perm=torch.arange(32))


def test_pipeline_chunk_plans():
    """Equal chunks for the all-to-all exchanges; the pull exchange cuts a
    small first chunk (its pull is the one not hidden under an attention)
    and attends the rest in one launch."""
    def plan(pipe):
        return [(s.start, s.stop) for s in pipe.chunk_slices()]
    assert plan(parallel.PipelinedHeadParallel(None, 2, 20, 16, chunks=2)) == [(0, 5), (5, 10)]
    assert plan(parallel.PipelinedHeadParallel(None, 2, 20, 16, chunks=2, peer_out=True)) == \
        [(0, 5), (5, 10)]
    assert plan(parallel.PipelinedHeadParallel(None, 2, 20, 16, chunks=2, peer_out=True,
                                               peer_in=True)) == [(0, 2), (2, 10)]
    assert plan(parallel.PipelinedHeadParallel(None, 8, 40, 16, peer_out=True,
                                               peer_in=True)) == [(0, 1), (1, 5)]
    assert plan(parallel.PipelinedHeadParallel(None, 2, 40, 16, peer_out=True, peer_in=True,
                                               pull_chunks=[4, 8, 8])) == [(0, 4), (4, 12),
                                                                           (12, 20)]
    # pull chunks without peer outputs do not apply
    assert plan(parallel.PipelinedHeadParallel(None, 2, 20, 16, chunks=2, peer_in=True)) == \
        [(0, 5), (5, 10)]
    for bad in ([3, 3], [0, 10], [11, -1]):
        with pytest.raises(ValueError):
            parallel.PipelinedHeadParallel(None, 2, 20, 16, peer_out=True, peer_in=True,
                                           pull_chunks=bad)


def test_keep_fraction_is_global():
    results = run_ranks(_keep)
    assert results[0] == results[1] == pytest.approx(16 / 64)


def test_plans():
    p = parallel.make_plan(8, 5, 40, batch=2)
    assert (p.cfg_groups, p.group_size, p.group_index, p.group_rank) == (2, 4, 1, 1)
    assert p.head_slice == slice(10, 20) and p.branches(2) == [1]
    p = parallel.make_plan(2, 1, 40, batch=2)
    assert p.group_size == 1 and p.branches(2) == [1] and p.head_slice == slice(0, 40)
    p = parallel.make_plan(1, 0, 40, batch=2)
    assert p.cfg_groups == 1 and p.branches(2) == [0, 1]
    p = parallel.make_plan(8, 3, 40, batch=2, split_cfg=False)
    assert p.group_size == 8 and p.head_slice == slice(15, 20)
    with pytest.raises(ValueError):
        parallel.make_plan(3, 0, 40, batch=1)
