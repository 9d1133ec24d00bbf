"""Head-parallel (Ulysses) execution of the routed attention across GPUs.

The reference runs on one device.  Routes, masses, CSR and attention are all
per head, so the path partitions by heads: a sequence-parallel caller holding
``[B, T/P, H, D]`` shards exchanges them with one all-to-all into head shards
``[B, T, H/P, D]``, runs the local pack -> attention -> unpack, and exchanges
the output back.  The only cross-head coupling of the reference is the
dense-dispatch keep fraction (``flex.py:473-493``), a mean over all heads,
which needs one integer all-reduce (``FlexReuseBackend(process_group=...)``).

With an even number of ranks the two CFG branches (the reference's two
batch-1 calls per denoising step) run on separate rank groups, which halves
the all-to-all group.  Collectives go through ``torch.distributed`` (NCCL on
GPUs, gloo on CPU for tests).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class ParallelPlan:
    """Placement of one attention layer's (branch, head) work on the ranks."""
    world: int
    rank: int
    cfg_groups: int           # 1 or 2 rank groups (one CFG branch each)
    group_size: int           # ranks sharing one branch (all-to-all width)
    group_index: int          # which branch group this rank belongs to
    group_rank: int           # rank within the group
    heads: int

    @property
    def heads_per_rank(self):
        return self.heads // self.group_size

    @property
    def head_slice(self):
        start = self.group_rank * self.heads_per_rank
        return slice(start, start + self.heads_per_rank)

    def branches(self, batch):
        """CFG branches (batch indices) this rank's group processes."""
        if self.cfg_groups == 1:
            return list(range(batch))
        per = math.ceil(batch / self.cfg_groups)
        return list(range(self.group_index * per, min(batch, (self.group_index + 1) * per)))


def make_plan(world, rank, heads, batch=2, split_cfg=True):
    cfg_groups = 2 if (split_cfg and batch >= 2 and world >= 2 and world % 2 == 0) else 1
    group_size = world // cfg_groups
    if heads % group_size:
        raise ValueError(f"{heads} heads do not split over {group_size} ranks")
    return ParallelPlan(world, rank, cfg_groups, group_size, rank // group_size,
                        rank % group_size, heads)


def exchange_group_options():
    """Process-group options for the head exchange: on NCCL, collectives on
    high-priority streams.  The attention fills every SM (one CTA per SM),
    so a collective issued under it gets SMs only as its CTAs retire; with
    higher priority the collective's CTAs take the next free SMs instead of
    waiting for the whole attention grid, and the exchange of chunk c + 1
    runs under chunk c's attention."""
    if dist.get_backend() != "nccl":
        return None
    opts = dist.ProcessGroupNCCL.Options()
    opts.is_high_priority_stream = True
    return opts


def new_groups(plan):
    """Create the exchange groups, one per CFG branch group (every rank calls
    this with the same plan); NCCL groups run on high-priority streams."""
    opts = exchange_group_options()
    mine = None
    for g in range(plan.cfg_groups):
        ranks = list(range(g * plan.group_size, (g + 1) * plan.group_size))
        pg = dist.new_group(ranks, pg_options=opts)
        if g == plan.group_index:
            mine = pg
    return mine


def seq_to_head(x, group, group_size):
    """``[B, T/P, H, D]`` sequence shard -> ``[B, T, H/P, D]`` head shard."""
    if group_size == 1:
        return x.contiguous()
    b, t_local, h, d = x.shape
    hp = h // group_size
    send = x.reshape(b, t_local, group_size, hp, d).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[src] holds tokens [src*T/P, (src+1)*T/P) of this rank's heads
    return recv.permute(1, 0, 2, 3, 4).reshape(b, group_size * t_local, hp, d)


def head_to_seq(x, group, group_size):
    """``[B, T, H/P, D]`` head shard -> ``[B, T/P, H, D]`` sequence shard."""
    if group_size == 1:
        return x.contiguous()
    b, t, hp, d = x.shape
    t_local = t // group_size
    send = x.reshape(b, group_size, t_local, hp, d).permute(1, 0, 2, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[src] holds this rank's tokens for the heads of rank src
    return recv.permute(1, 2, 0, 3, 4).reshape(b, t_local, group_size * hp, d)


class CudaRows:
    """Row moves of the exchange on the GPU: ``gather`` is ``kernels.reorder_rows``
    (``out[b, i] = x[b, perm[i]]``), ``scatter`` is
    ``kernels.gather_scatter_rows`` (``dst[b, off + dst_rows[i]] = src[b, src_rows[i]]``)."""

    @staticmethod
    def gather(tensors, perm):
        from . import kernels
        return kernels.reorder_rows(tensors, perm)

    @staticmethod
    def scatter(srcs, dsts, src_rows, dst_rows, dst_offsets=None):
        from . import kernels
        kernels.gather_scatter_rows(srcs, dsts, src_rows, dst_rows, dst_offsets)


class _Tables:
    """Row maps of one exchange shape, built once on the CPU, cached per device."""

    def __init__(self, builders):
        self._builders = builders
        self._cpu = {name: fn().to(torch.int32) for name, fn in builders.items()}
        self._dev = {}

    def get(self, name, device):
        key = (name, device)
        if key not in self._dev:
            self._dev[key] = self._cpu[name].to(device)
        return self._dev[key]


def _send_maps(P, tl, groups):
    """For a sequence shard ``[tl, P * groups, rowsz]`` (rows of one head
    group): the source row and send-buffer row of every (destination rank p,
    token i) for head group ``g`` of each rank, the send buffer being
    ``[P, 3, tl, rowsz]`` with Q, K, V at row offsets 0, tl, 2 tl."""
    p = torch.arange(P)[:, None]
    i = torch.arange(tl)[None, :]
    dst = (p * 3 * tl + i).reshape(-1)

    def src(g):
        return ((i * P + p) * groups + g).reshape(-1)
    return src, dst


def head_parallel_attention(q, k, v, attend, group, group_size, rows=None):
    """Run ``attend(q, k, v) -> out`` on head shards of sequence-sharded inputs.

    ``q, k, v``: ``[B, T/P, H, D]``; ``attend`` receives ``[B, T, H/P, D]``
    tensors and returns the same shape (for example pack -> block-sparse
    attention over this rank's heads' CSR routes -> unpack).  With batch 1 the
    send buffer is written by one row gather (no concatenation or transpose
    copies), the received rows are gathered into token order, and the output
    rows are scattered back into ``[T/P, H, D]``; ``rows`` supplies those row
    moves (``CudaRows`` by default).
    """
    if group_size == 1:
        return attend(q, k, v)
    b, tl, h, d = q.shape
    if b != 1:
        stacked = torch.cat([q, k, v], 0)             # one exchange for Q, K and V
        heads = seq_to_head(stacked, group, group_size)
        out = attend(heads[:b], heads[b:2 * b], heads[2 * b:])
        return head_to_seq(out, group, group_size)
    rows = rows or CudaRows
    P = group_size
    hp = h // P
    T = P * tl
    src_of, dst = _send_maps(P, tl, 1)
    src = src_of(0)
    send = torch.empty((P * 3 * tl, hp, d), dtype=q.dtype, device=q.device)
    flat = [x.contiguous().view(1, tl * P, hp, d) for x in (q, k, v)]
    rows.scatter(flat, [send[None]] * 3, src.to(q.device, torch.int32),
                 dst.to(q.device, torch.int32), dst_offsets=[0, tl, 2 * tl])
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv = [src rank p, q|k|v, tl, hp, d]: token p * tl + i of tensor t is
    # row (p * 3 + t) * tl + i
    g = torch.arange(T)
    order = ((g // tl) * 3 * tl + g % tl).to(q.device, torch.int32)
    span = (3 * P - 2) * tl
    r = recv[None]
    qh, kh, vh = rows.gather([r[:, t * tl:t * tl + span] for t in range(3)], order)
    out_h = attend(qh, kh, vh).contiguous()
    orecv = torch.empty_like(out_h)
    dist.all_to_all_single(orecv, out_h, group=group)
    # orecv = [src rank p, tl, hp, d] -> out [tl, P, hp, d]: row p*tl + i -> i*P + p
    out = torch.empty_like(q)
    rows.scatter([orecv.view(1, T, hp, d)], [out.view(1, T, hp, d)],
                 torch.arange(T, dtype=torch.int32, device=q.device), src.to(q.device, torch.int32))
    return out


# Allocations of other processes mapped into this one, by IPC handle: a
# handle (one cudaMalloc segment) is opened once per process and reused.
_IPC_BASES: dict = {}


class PeerShards:
    """This rank's shard (``shape``: the output ``[T/P, H, D]``, or the
    inputs ``[3, T/P, H, D]``) and every group rank's shard mapped into this
    process (CUDA IPC, exchanged once over the group), so a kernel can store
    each output row into the rank that holds its token, or pull each input
    row from it.  ``ptrs[d]`` is rank d's shard (this rank's own for d = its
    rank).  ``ready`` is the same on every rank: False when any rank could
    not export or map a shard (``error`` holds this rank's cause, if any)."""

    def __init__(self, group, group_size, shape, dtype, device):
        from . import kernels
        self.local = torch.empty(shape, dtype=dtype, device=device)
        self.ptrs = []
        self.error = None
        try:
            handle, offset = kernels.ipc_export(self.local)
        except RuntimeError as exc:          # e.g. memory the runtime cannot export
            self.error = exc
            handle, offset = bytes(64), 0
        mine = torch.tensor(list(handle) + list(int(offset).to_bytes(8, "little")),
                            dtype=torch.uint8, device=device)
        every = [torch.empty_like(mine) for _ in range(group_size)]
        dist.all_gather(every, mine, group=group)
        me = dist.get_rank(group)
        for r, t in enumerate(every):
            if self.error is not None:
                break
            if r == me:
                self.ptrs.append(self.local.data_ptr())
                continue
            raw = bytes(t.cpu().tolist())
            off = int.from_bytes(raw[64:], "little")
            base = _IPC_BASES.get(raw[:64])
            try:
                if base is None:
                    base = kernels.ipc_import(raw[:64], 0)
                    _IPC_BASES[raw[:64]] = base
            except RuntimeError as exc:
                self.error = exc
                break
            self.ptrs.append(base + off)
        # every rank takes the same exchange: peer stores only if all mapped
        ok = torch.tensor([0 if self.error is not None else 1], dtype=torch.int32, device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        self.ready = bool(ok.item())


def pipeline_chunks(heads_per_rank):
    """Head chunks per rank for ``PipelinedHeadParallel``: 4, 2, 5 or 3 chunks
    of at least 4 heads each, else 1.  Smaller chunks hide more of the
    exchange but each chunk's attention launch then has few waves of CTAs
    (2-head chunks at 8 GPUs: 900 CTAs, 6.1 waves on 148 SMs) and its tail
    costs more than the exchange it hides (measured: 10.1-10.8 ms of
    attention per rank with 2-head chunks against 9.3-9.7 ms with 5-head
    chunks)."""
    for c in (4, 2, 5, 3):
        if heads_per_rank % c == 0 and heads_per_rank // c >= 4:
            return c
    return 1


class PipelinedHeadParallel:
    """Ulysses exchange in head chunks, overlapped with the attention.

    For one CFG branch (batch 1) of sequence shards ``[1, T/P, H, D]``: this
    rank's ``H/P`` heads are split into ``chunks`` groups.  Every chunk's send
    buffer ``[P, q|k|v, T/P, hc, D]`` is written by one row-gather launch and
    its input all-to-all issued up front on NCCL's stream.  Chunk c's packed
    Q/K/V are gathered straight from its receive buffer (the pack permutation
    remapped onto the receive layout), ``attend`` runs on them and stores its
    output rows in token order - the send layout of the output all-to-all -
    which is sent while the next chunk computes; each received output chunk
    is scattered into ``[T/P, H, D]`` by one launch.  Only the first chunk's
    input exchange and the last chunk's output exchange stay exposed.

    ``attend(qp, kp, vp, chunk, out, out_rows)`` gets ``[1, T, hc, D]`` tensors
    in pack order and either writes the output to token ``out_rows[i]`` of
    ``out`` (``[1, T, hc, D]``; ``out_rows`` is None without a permutation) and
    returns None - the block-sparse kernel's folded unpack - or returns the
    output in pack order.  ``rows`` supplies the row moves (``CudaRows``).

    ``peer_out`` (CUDA): no output all-to-all.  Every rank's output shard is
    mapped into the others (``PeerShards``) and ``attend`` is called with
    ``out=None`` and ``peers=`` a ``kernels.PeerRows`` for the chunk's heads:
    the attention kernel stores each row into the rank holding its token
    (``kernels.block_sparse_attention_peers``), so the output exchange runs
    inside the attention.  One small all-reduce then joins the ranks before
    the shard is read.  The next call's first input exchange cannot complete
    before every rank has started that call, so no rank stores into a shard
    its owner is still reading.

    ``peer_in`` (with ``peer_out``): no input all-to-all either.  Every rank's
    Q/K/V shard sits in a mapped buffer (``input_buffers``; other inputs are
    copied there), and each chunk's packed rows are pulled from the ranks'
    shards over peer memory (``kernels.pull_rows``) on a high-priority side
    stream while earlier chunks attend.  One all-reduce before the pulls
    (every shard written) and one after the attention (every store done)
    are the only collectives.  Pull chunks need no all-to-all layout, so
    they are cut by ``pull_chunks`` (head counts; default a fifth of the
    rank's heads, at least one, then the rest): only the first chunk's pull
    waits in front of an attention.  ``chunk_slices()`` gives the local head
    range of every chunk of the exchange in effect.  If any rank cannot map
    the shards, every rank takes the all-to-all exchange (equal chunks).
    """

    def __init__(self, group, group_size, heads, tokens_local, perm=None, inverse=None,
                 chunks=None, rows=None, peer_out=False, peer_in=False, pull_chunks=None):
        if heads % group_size:
            raise ValueError(f"{heads} heads do not split over {group_size} ranks")
        self.group = group
        self.P = group_size
        self.hp = heads // group_size
        self.chunks = chunks or pipeline_chunks(self.hp)
        if self.hp % self.chunks:
            raise ValueError(f"{self.hp} heads per rank do not split into {self.chunks} chunks")
        self.hc = self.hp // self.chunks
        self.tl = tokens_local
        tokens = tokens_local * group_size
        if (inverse is None) != (perm is None):
            raise ValueError("give both perm and inverse, or neither")
        perm = (torch.arange(tokens, dtype=torch.int64) if perm is None
                else torch.as_tensor(perm).to("cpu", torch.int64))
        if perm.numel() != tokens:
            raise ValueError("perm must cover the whole sequence")
        self.has_perm = inverse is not None
        P, tl, C = self.P, self.tl, self.chunks
        src_of, dst = _send_maps(P, tl, C)
        src, local = perm // tl, perm % tl
        builders = {"recv_perm": lambda: src * 3 * tl + local,   # row of token perm[i], tensor 0
                    "send_dst": lambda: dst,
                    "out_src": lambda: torch.arange(P * tl),
                    "perm": lambda: perm}
        for c in range(C):
            builders[f"send_src{c}"] = (lambda c=c: src_of(c))
        if inverse is not None:
            inv = torch.as_tensor(inverse).to("cpu", torch.int64)
            builders["inverse"] = lambda: inv
        self.tables = _Tables(builders)
        self.rows = rows or CudaRows
        self.peer_out = peer_out
        self.peer_in = peer_in and peer_out
        # Pull mode cuts the heads freely (no all-to-all layout): a small
        # first chunk, whose pull is the only one not hidden under an
        # attention, then the rest in one launch.
        if pull_chunks is None:
            first = max(1, self.hp // 5)
            pull_chunks = [first, self.hp - first] if self.hp > first else [self.hp]
        if sum(pull_chunks) != self.hp or min(pull_chunks) < 1:
            raise ValueError("pull_chunks must be positive head counts summing to the rank's heads")
        self.pull_chunks = list(pull_chunks)
        self.peer_error = None
        self._shards = {}
        self._in_shards = {}
        self._pull = {}

    def chunk_slices(self):
        """This rank's local head range of every chunk, in call order, for the
        exchange in effect (pull chunks with ``peer_in``, else equal ones)."""
        sizes = self.pull_chunks if self.peer_in else [self.hc] * self.chunks
        out, start = [], 0
        for n in sizes:
            out.append(slice(start, start + n))
            start += n
        return out

    def input_buffers(self, device, dtype, head_dim):
        """With ``peer_in``: (q, k, v) ``[1, T/P, H, D]`` views of this rank's
        mapped input shard; inputs written there are not copied by the call."""
        ins = self._input_shards(torch.device(device), dtype, self.hp * self.P, head_dim)
        return tuple(ins.local[x][None] for x in range(3))

    def _input_shards(self, device, dtype, h, d):
        key = (device, dtype, d)
        ins = self._in_shards.get(key)
        if ins is None:
            ins = self._in_shards[key] = PeerShards(self.group, self.P, (3, self.tl, h, d),
                                                    dtype, device)
        return ins

    def _output_shards(self, device, dtype, h, d):
        key = (device, dtype, d)
        shards = self._shards.get(key)
        if shards is None:
            shards = self._shards[key] = PeerShards(self.group, self.P, (self.tl, h, d), dtype,
                                                    device)
        return shards

    def _pull_call(self, q, k, v, attend):
        """Input exchange by pulls over peer memory, output by the attention's
        stores: no NCCL all-to-all.  The caller's shards go into this rank's
        mapped input shard (unless already there); after one all-reduce every
        rank's inputs are in place, and a high-priority side stream pulls each
        chunk's packed rows (``kernels.pull_rows``) while earlier chunks
        attend."""
        from . import kernels
        from .kernels import PeerRows
        _, tl, h, d = q.shape
        dev = q.device
        ins = self._input_shards(dev, q.dtype, h, d)
        outs = self._output_shards(dev, q.dtype, h, d)
        if not (ins.ready and outs.ready):
            self.peer_in = self.peer_out = False
            self.peer_error = ins.error or outs.error
            return None
        for x, t in enumerate((q, k, v)):
            if t.data_ptr() != ins.local[x].data_ptr():
                ins.local[x].copy_(t[0])
        # every rank's inputs are in its shard before any rank pulls
        joined = torch.zeros(1, dtype=torch.float32, device=dev)
        dist.all_reduce(joined, group=self.group)
        slices = self.chunk_slices()
        pull_key = (dev, q.dtype, d)     # pull buffers per device, dtype and head size
        state = self._pull.get(pull_key)
        if state is None:
            side = torch.cuda.Stream(device=dev, priority=-1)
            bufs = [[torch.empty((1, tl * self.P, sl.stop - sl.start, d), dtype=q.dtype,
                                 device=dev) for _ in range(3)] for sl in slices]
            state = self._pull[pull_key] = (side, bufs)
        side, bufs = state
        cur = torch.cuda.current_stream(dev)
        ready = torch.cuda.Event()
        ready.record(cur)
        side.wait_event(ready)
        me = dist.get_rank(self.group)
        perm = self.tables.get("perm", dev) if self.has_perm else None
        pulled = []
        with torch.cuda.stream(side):
            for c, sl in enumerate(slices):
                kernels.pull_rows(ins.ptrs, tl, h * d * q.element_size(),
                                  tl * h * d * q.element_size(),
                                  (me * self.hp + sl.start) * d * q.element_size(), bufs[c],
                                  perm)
                e = torch.cuda.Event()
                e.record(side)
                pulled.append(e)
        mine = PeerRows(outs.ptrs, tl, h * d, d).shifted(me * self.hp)
        for c, sl in enumerate(slices):
            cur.wait_event(pulled[c])
            attend(*bufs[c], c, None, perm, peers=mine.shifted(sl.start))
        # every rank's stores into this shard are done once all ranks get here
        dist.all_reduce(joined, group=self.group)
        return outs.local.clone().view(1, tl, h, d)

    def __call__(self, q, k, v, attend):
        b, tl, h, d = q.shape
        if b != 1 or tl != self.tl or h != self.hp * self.P:
            raise ValueError("PipelinedHeadParallel takes [1, T/P, H, D] shards of one branch")
        if self.peer_in:
            out = self._pull_call(q, k, v, attend)
            if out is not None:
                return out
        P, hc, C = self.P, self.hc, self.chunks
        T = P * tl
        dev = q.device
        tab = lambda name: self.tables.get(name, dev)  # noqa: E731
        flat = [x.contiguous().view(1, tl * P * C, hc, d) for x in (q, k, v)]
        send = torch.empty((C, P * 3 * tl, hc, d), dtype=q.dtype, device=dev)
        recv = torch.empty_like(send)
        inputs = []
        for c in range(C):
            self.rows.scatter(flat, [send[c][None]] * 3, tab(f"send_src{c}"), tab("send_dst"),
                              dst_offsets=[0, tl, 2 * tl])
            inputs.append(dist.all_to_all_single(recv[c], send[c], group=self.group,
                                                 async_op=True))
        span = (3 * P - 2) * tl
        out_rows = tab("perm") if self.has_perm else None
        if self.peer_out:
            out = self._peer_call(q, recv, inputs, attend, out_rows, span)
            if out is not None:
                return out
        out_send = torch.empty((C, T, hc, d), dtype=q.dtype, device=dev)
        orecv = torch.empty_like(out_send)
        outputs = []
        for c in range(C):
            inputs[c].wait()
            r = recv[c][None]
            qp, kp, vp = self.rows.gather([r[:, t * tl:t * tl + span] for t in range(3)],
                                          tab("recv_perm"))
            res = attend(qp, kp, vp, c, out_send[c][None], out_rows)
            if res is not None:          # output in pack order: unpack it here
                if self.has_perm:
                    self.rows.scatter([res.contiguous()], [out_send[c][None]], tab("out_src"),
                                      tab("perm"))
                else:
                    out_send[c].copy_(res[0])
            outputs.append(dist.all_to_all_single(orecv[c], out_send[c], group=self.group,
                                                  async_op=True))
        out = torch.empty_like(q)
        dst = out.view(1, tl * P * C, hc, d)
        for c in range(C):
            outputs[c].wait()
            self.rows.scatter([orecv[c][None]], [dst], tab("out_src"), tab(f"send_src{c}"))
        return out

    def _peer_call(self, q, recv, inputs, attend, out_rows, span):
        from .kernels import PeerRows
        _, tl, h, d = q.shape
        shards = self._output_shards(q.device, q.dtype, h, d)
        if not shards.ready:
            # some rank could not map the shards: every rank exchanges by NCCL
            self.peer_out = False
            self.peer_error = shards.error
            return None
        me = dist.get_rank(self.group)
        mine = PeerRows(shards.ptrs, tl, h * d, d).shifted(me * self.hp)
        for c in range(self.chunks):
            inputs[c].wait()
            r = recv[c][None]
            qp, kp, vp = self.rows.gather([r[:, t * tl:t * tl + span] for t in range(3)],
                                          self.tables.get("recv_perm", q.device))
            attend(qp, kp, vp, c, None, out_rows, peers=mine.shifted(c * self.hc))
        # every rank's stores into this shard are done once all ranks get here
        joined = torch.zeros(1, dtype=torch.float32, device=q.device)
        dist.all_reduce(joined, group=self.group)
        return shards.local.clone().view(1, tl, h, d)


def all_reduce_count(count, group=None):
    """Sum an integer count over the group (the dense-dispatch keep numerator)."""
    t = count.clone() if torch.is_tensor(count) else torch.tensor([int(count)])
    dist.all_reduce(t, group=group)
    return t
