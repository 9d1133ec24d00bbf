"""Head-parallel exchange on real GPUs (NCCL), when the box has two or more.

Two ranks hold sequence shards of one branch; every exchange path - the
unchunked ``head_parallel_attention``, the chunked ``PipelinedHeadParallel``
with the routed kernel storing into the output all-to-all's send buffer or
straight into the ranks' output shards over peer memory (twice in a row),
with the inputs pulled from the ranks' mapped shards as well, and
the public ``FlexReuseBackend.head_parallel`` on a reuse call - must give the
single-GPU result on every row of the rank's shard.  Skipped with fewer than two GPUs; the host-side
layout logic is covered on CPU by tests/test_parallel_gloo.py.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import torch.distributed as dist
    from datetime import timedelta

    from dit_sparse_atten_b200 import _native, kernels, parallel
    from dit_sparse_atten_b200.context import set_routing_context
    from dit_sparse_atten_b200.flex import FlexReuseBackend, FlexReuseConfig
    from dit_sparse_atten_b200.spatial import build_spatial_layout

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        grid, H = (4, 16, 32), 8                  # 2,048 tokens, 16 route blocks
        T = grid[0] * grid[1] * grid[2]
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn((1, T, H, 128), generator=g).to(torch.bfloat16).to(dev)
                   for _ in range(3))
        route = torch.rand((H, 16, 16), generator=g) < 0.5
        route[..., 0] = True
        lay = build_spatial_layout(grid, 128)
        counts, indices = kernels.pack_boolean_rows(route.to(dev))
        # single-GPU reference: pack, routed attention, unpack
        qp, kp, vp = lay.reorder_qkv(q, k, v)
        ref = lay.restore(kernels.block_sparse_attention(qp, kp, vp, counts, indices))
        tl = T // world
        sl = slice(rank * tl, (rank + 1) * tl)
        hp = H // world
        hs = slice(rank * hp, (rank + 1) * hp)
        c_loc, i_loc = counts[hs].contiguous(), indices[hs].contiguous()

        def attend(qh, kh, vh):
            a, b_, c = lay.reorder_qkv(qh, kh, vh)
            return kernels.block_sparse_attention(a, b_, c, c_loc, i_loc,
                                                  out_rows=lay.permutation(dev))

        out = parallel.head_parallel_attention(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                               v[:, sl].contiguous(), attend,
                                               dist.group.WORLD, world)
        errs = [float((out.float() - ref[:, sl].float()).abs().max())]
        pipe = parallel.PipelinedHeadParallel(dist.group.WORLD, world, H, tl,
                                              perm=lay.permutation_cpu, inverse=lay.inverse_cpu,
                                              chunks=2)

        def attend_for(pipe_):
            # chunk c's local heads under the chunk plan of pipe_'s exchange
            def attend_chunk(qp_, kp_, vp_, c, out_c, out_rows, peers=None):
                cs = pipe_.chunk_slices()[c]
                if peers is not None:
                    kernels.block_sparse_attention_peers(qp_, kp_, vp_, c_loc[cs].contiguous(),
                                                         i_loc[cs].contiguous(), peers,
                                                         out_rows=out_rows)
                    return
                kernels.block_sparse_attention(qp_, kp_, vp_, c_loc[cs].contiguous(),
                                               i_loc[cs].contiguous(), out=out_c,
                                               out_rows=out_rows)
            return attend_chunk

        out2 = pipe(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(),
                    attend_for(pipe))
        # the output exchange inside the attention: stores into the ranks'
        # shards over peer memory, twice in a row (the second call stores into
        # shards the first call's owners have read)
        pipe_o = parallel.PipelinedHeadParallel(dist.group.WORLD, world, H, tl,
                                                perm=lay.permutation_cpu,
                                                inverse=lay.inverse_cpu, chunks=2, peer_out=True)
        shard = [x[:, sl].contiguous() for x in (q, k, v)]
        out4 = pipe_o(*shard, attend_for(pipe_o))
        out5 = pipe_o(*[x.flip(1).contiguous() for x in shard], attend_for(pipe_o))
        out4b = pipe_o(*shard, attend_for(pipe_o))
        # and the input exchange as pulls from the ranks' mapped input shards:
        # copied in, then already in place
        pipe_p = parallel.PipelinedHeadParallel(dist.group.WORLD, world, H, tl,
                                                perm=lay.permutation_cpu,
                                                inverse=lay.inverse_cpu, chunks=2, peer_out=True,
                                                peer_in=True)
        # pulls are cut unevenly: a one-head first chunk, then the rest
        assert [s_.stop - s_.start for s_ in pipe_p.chunk_slices()] == [1, hp - 1]
        out6 = pipe_p(*shard, attend_for(pipe_p))
        bufs = pipe_p.input_buffers(dev, q.dtype, 128)
        for dst_t, src_t in zip(bufs, shard):
            dst_t.copy_(src_t)
        out7 = pipe_p(*bufs, attend_for(pipe_p))
        assert pipe_p.peer_in and pipe_o.peer_out and not pipe_o.peer_in
        # the public API: FlexReuseBackend.head_parallel on a reuse call
        backend = FlexReuseBackend(FlexReuseConfig(spatial_reorder=True))
        backend.install_route(route[hs].to(dev), attention_id=1, branch=0, tokens=T, heads=hp,
                              head_dim=128, device=dev, grid=grid)
        set_routing_context(attention_id=1, step=1, branch=0, grid=grid)
        out3 = backend.head_parallel(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                     v[:, sl].contiguous(), dist.group.WORLD, world, chunks=2)
        torch.cuda.synchronize()
        _native.check_device_errors()
        assert backend.pipelines and backend.phase_counts["sparse_reuse"] == 1
        errs.append(float((out2.float() - ref[:, sl].float()).abs().max()))
        errs.append(float((out3.float() - ref[:, sl].float()).abs().max()))
        errs.append(float((out4.float() - ref[:, sl].float()).abs().max()))
        errs.append(float((out4b.float() - ref[:, sl].float()).abs().max()))
        errs.append(float((out6.float() - ref[:, sl].float()).abs().max()))
        errs.append(float((out7.float() - ref[:, sl].float()).abs().max()))
        assert not torch.equal(out5, out4)
        assert backend.pipelines and all(p.peer_out for p in backend.pipelines.values())
        queue.put((rank, errs))
    except Exception as exc:
        queue.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_exchange_paths_match_single_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, errs in results.items():
        assert not isinstance(errs, str), errs
        # the same kernels on the same rows: the exchange must not change a bit
        assert errs == [0.0] * 7, (rank, errs)
