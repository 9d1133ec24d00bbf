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


def new_groups(plan):
    """Create the CFG rank groups (every rank calls this with the same plan)."""
    if plan.cfg_groups == 1:
        return dist.group.WORLD
    mine = None
    for g in range(plan.cfg_groups):
        ranks = list(range(g * plan.group_size, (g + 1) * plan.group_size))
        pg = dist.new_group(ranks)
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


def head_parallel_attention(q, k, v, attend, group, group_size):
    """Run ``attend(q, k, v) -> out`` on head shards of sequence-sharded inputs.

    ``q, k, v``: ``[B, T/P, H, D]``; ``attend`` receives ``[B, T, H/P, D]``
    tensors and returns the same shape (for example pack -> block-sparse
    attention over this rank's heads' CSR routes -> unpack).
    """
    stacked = torch.cat([q, k, v], 0)             # one exchange for Q, K and V
    heads = seq_to_head(stacked, group, group_size)
    b = q.shape[0]
    out = attend(heads[:b], heads[b:2 * b], heads[2 * b:])
    return head_to_seq(out, group, group_size)


def pipeline_chunks(heads_per_rank):
    """Head chunks per rank for ``PipelinedHeadParallel``: 4, 2, 5 or 3 chunks
    of at least 4 heads each (enough attention per chunk to hide the next
    chunk's exchange), else 1."""
    for c in (4, 2, 5, 3):
        if heads_per_rank % c == 0 and heads_per_rank // c >= 4:
            return c
    return 1


class PipelinedHeadParallel:
    """Ulysses exchange in head chunks, overlapped with the attention.

    For one CFG branch (batch 1) of sequence shards ``[1, T/P, H, D]``: this
    rank's ``H/P`` heads are split into ``chunks`` groups.  The input
    all-to-all of every chunk is issued up front on NCCL's stream; chunk c's
    packed Q/K/V are gathered straight from its receive buffer (no
    concatenation or transpose copies: the pack permutation is remapped onto
    the receive layout ``[src rank, q|k|v, T/P, heads, D]``), ``attend`` runs
    on them, the result is restored to token order - which is already the
    send layout of the output all-to-all - and sent back while the next chunk
    computes.  Only the first chunk's input exchange and the last chunk's
    output exchange stay exposed.

    ``attend(qp, kp, vp, chunk) -> out_p`` takes and returns ``[1, T, hc, D]``
    tensors in pack order (for example the routed attention over the chunk's
    heads' CSR).  ``gather(tensors, perm)`` is the row gather
    (``kernels.reorder_rows`` on GPUs; CPU tests pass an ``index_select``).
    """

    def __init__(self, group, group_size, heads, tokens_local, perm=None, inverse=None,
                 chunks=None, gather=None):
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
        src, local = perm // tokens_local, perm % tokens_local
        # row of token perm[i] of tensor 0 in the receive buffer viewed as
        # [P * 3 * T/P] rows; tensor t starts t * T/P rows later
        self._src_perm = (src * 3 * tokens_local + local).to(torch.int32)
        self._inverse = None if inverse is None else torch.as_tensor(inverse).to(torch.int32)
        self._dev = {}
        if gather is None:
            from . import kernels
            gather = kernels.reorder_rows
        self.gather = gather

    def _device_tables(self, device):
        if device not in self._dev:
            self._dev[device] = (self._src_perm.to(device),
                                 None if self._inverse is None else self._inverse.to(device))
        return self._dev[device]

    def __call__(self, q, k, v, attend):
        b, tl, h, d = q.shape
        if b != 1 or tl != self.tl or h != self.hp * self.P:
            raise ValueError("PipelinedHeadParallel takes [1, T/P, H, D] shards of one branch")
        P, hp, hc, C = self.P, self.hp, self.hc, self.chunks
        src_perm, inverse = self._device_tables(q.device)
        send = torch.empty((C, P, 3, tl, hc, d), dtype=q.dtype, device=q.device)
        recv = torch.empty_like(send)
        inputs = []
        for c in range(C):
            for t, x in enumerate((q, k, v)):
                send[c, :, t].copy_(x[0].view(tl, P, hp, d)[:, :, c * hc:(c + 1) * hc]
                                    .permute(1, 0, 2, 3))
            inputs.append(dist.all_to_all_single(recv[c], send[c], group=self.group,
                                                 async_op=True))
        span = (3 * P - 2) * tl
        outputs, sent = [], []
        orecv = torch.empty((C, P, tl, hc, d), dtype=q.dtype, device=q.device)
        for c in range(C):
            inputs[c].wait()
            flat = recv[c].view(1, P * 3 * tl, hc, d)
            qp, kp, vp = self.gather([flat[:, t * tl:t * tl + span] for t in range(3)], src_perm)
            out_p = attend(qp, kp, vp, c)
            out_c = out_p if inverse is None else self.gather([out_p], inverse)[0]
            sent.append(out_c)
            outputs.append(dist.all_to_all_single(orecv[c], out_c.view(P, tl, hc, d),
                                                  group=self.group, async_op=True))
        out = torch.empty_like(q)
        for c in range(C):
            outputs[c].wait()
            out[0].view(tl, P, hp, d)[:, :, c * hc:(c + 1) * hc].copy_(
                orecv[c].permute(1, 0, 2, 3))
        return out


def all_reduce_count(count, group=None):
    """Sum an integer count over the group (the dense-dispatch keep numerator)."""
    t = count.clone() if torch.is_tensor(count) else torch.tensor([int(count)])
    dist.all_reduce(t, group=group)
    return t
