"""torch-facing wrappers of the C ABI (one function per entry point of include/bsa.h).

Each wrapper checks shapes/dtypes, allocates the outputs with torch on the
inputs' device, and enqueues the kernel on the current CUDA stream.  Inputs
must be CUDA tensors; nothing here has a CPU path.
"""

from __future__ import annotations

import ctypes
import functools
import math
from typing import NamedTuple, Sequence

import torch

from . import _native

HEAD_DIM = 128


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "the routed block-sparse path runs only on CUDA tensors "
                f"(got a {t.device} tensor); it has no CPU implementation")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("all tensors must be on the same device")
    return device


def _stream(device) -> int:
    return _native.stream_handle(device)


# ----------------------------------------------------------------------------
# (c) reorder
# ----------------------------------------------------------------------------

def reorder_rows(tensors: Sequence[torch.Tensor], perm: torch.Tensor,
                 tokens_out: int | None = None) -> tuple:
    """Gather token rows: ``out[b, i] = x[b, perm[i]]`` for 1-3 tensors ``[B, T, ...]``.

    Same result as ``x.index_select(1, perm)`` (reference ``spatial.py:82-93``).
    """
    tensors = [t.contiguous() for t in tensors]
    if not 1 <= len(tensors) <= 3:
        raise ValueError("reorder_rows takes one to three tensors")
    first = tensors[0]
    device = _require_cuda(*tensors, perm)
    if any(t.shape != first.shape or t.dtype != first.dtype for t in tensors):
        raise ValueError("tensors must share shape and dtype")
    if first.dim() < 2:
        raise ValueError("tensors must have a batch and a token axis")
    perm = perm.to(device=device, dtype=torch.int32).contiguous()
    if perm.dim() != 1:
        raise ValueError("perm must be one-dimensional")
    tokens_out = perm.numel() if tokens_out is None else tokens_out
    batch, tokens_in = first.shape[0], first.shape[1]
    row_bytes = first[0, 0].numel() * first.element_size() if tokens_in else 0
    outs = [torch.empty((batch, tokens_out) + tuple(first.shape[2:]), dtype=first.dtype,
                        device=device) for _ in tensors]
    if batch == 0 or tokens_out == 0 or row_bytes == 0:
        return tuple(outs)
    n = len(tensors)
    src = (ctypes.c_void_p * 3)(*([t.data_ptr() for t in tensors] + [0] * (3 - n)))
    dst = (ctypes.c_void_p * 3)(*([t.data_ptr() for t in outs] + [0] * (3 - n)))
    _native.call("bsa_reorder_rows", n, src, dst, perm.data_ptr(), batch, tokens_out,
                 tokens_in, row_bytes, _native.err_word(device).data_ptr(), _stream(device))
    return tuple(outs)


def gather_scatter_rows(srcs: Sequence[torch.Tensor], dsts: Sequence[torch.Tensor],
                        src_rows: torch.Tensor, dst_rows: torch.Tensor,
                        dst_offsets: Sequence[int] | None = None) -> None:
    """``dst[t][b, off_t + dst_rows[i]] = src[t][b, src_rows[i]]`` for 1-3 pairs
    of ``[B, tokens, ...]`` tensors with equal row sizes
    (``bsa_gather_scatter_rows``): the row moves of the head-parallel exchange.
    ``dsts`` are written in place and must be contiguous; ``dst_offsets``
    (rows, default 0) lets several sources land in one destination buffer."""
    if not 1 <= len(srcs) == len(dsts) <= 3:
        raise ValueError("one to three source/destination pairs")
    offsets = list(dst_offsets) if dst_offsets is not None else [0] * len(dsts)
    if len(offsets) != len(dsts) or any(o < 0 for o in offsets):
        raise ValueError("one non-negative row offset per destination")
    device = _require_cuda(*srcs, *dsts, src_rows, dst_rows)
    first, out0 = srcs[0], dsts[0]
    if any(t.shape[0] != first.shape[0] for t in (*srcs, *dsts)):
        raise ValueError("sources and destinations must share the batch size")
    row_bytes = first[0, 0].numel() * first.element_size()
    if any(t[0, 0].numel() * t.element_size() != row_bytes for t in (*srcs, *dsts)):
        raise ValueError("sources and destinations must share the row size")
    if any(not t.is_contiguous() for t in (*srcs, *dsts)):
        raise ValueError("gather_scatter_rows needs contiguous tensors")
    src_rows = src_rows.to(device=device, dtype=torch.int32).contiguous()
    dst_rows = dst_rows.to(device=device, dtype=torch.int32).contiguous()
    if src_rows.numel() != dst_rows.numel():
        raise ValueError("src_rows and dst_rows must have equal lengths")
    n = len(srcs)
    if src_rows.numel() == 0 or first.shape[0] == 0:
        return
    if any(o > t.shape[1] for o, t in zip(offsets, dsts)):
        raise ValueError("row offset past the destination")
    if any(offsets) and first.shape[0] != 1:
        raise ValueError("row offsets need batch 1")
    # rows addressable from every destination's offset base
    tokens_dst = min(t.shape[1] - o for o, t in zip(offsets, dsts))
    src = (ctypes.c_void_p * 3)(*([t.data_ptr() for t in srcs] + [0] * (3 - n)))
    dst = (ctypes.c_void_p * 3)(*([t.data_ptr() + o * row_bytes for o, t in zip(offsets, dsts)]
                                  + [0] * (3 - n)))
    _native.call("bsa_gather_scatter_rows", n, src, dst, src_rows.data_ptr(), dst_rows.data_ptr(),
                 first.shape[0], src_rows.numel(), first.shape[1], tokens_dst, row_bytes,
                 _native.err_word(device).data_ptr(), _stream(device))


# ----------------------------------------------------------------------------
# (b) route: sampling, mass, selection, CSR
# ----------------------------------------------------------------------------

@functools.lru_cache(maxsize=64)
def _sample_tables(tokens: int, block: int, samples: int):
    """Sample token ids and per-block key weights (reference ``flex.py:222-237``)."""
    blocks = math.ceil(tokens / block)
    block_ids = torch.arange(blocks)
    sizes = (tokens - block_ids * block).clamp(max=block)
    sample_ids = torch.arange(samples)
    local = torch.div((2 * sample_ids + 1)[None] * sizes[:, None], 2 * samples,
                      rounding_mode="floor").clamp_max(sizes[:, None] - 1)
    ids = (block_ids[:, None] * block + local).reshape(-1).to(torch.int32)
    bias = (sizes.float() / samples).log()
    return ids, bias


@functools.lru_cache(maxsize=64)
def _device_sample_tables(tokens: int, block: int, samples: int, device: torch.device):
    ids, bias = _sample_tables(tokens, block, samples)
    return ids.to(device), bias.to(device)


def sampled_block_mass(q: torch.Tensor, k: torch.Tensor, block: int = 128, samples: int = 2,
                       scale: float | None = None, round_bf16: bool = True,
                       one_pass: bool = True) -> torch.Tensor:
    """Sampled block mass ``[B, H, Qb, Qb]`` fp32 from bf16 ``q, k [B, T, H, D]``.

    Reference ``flex.py:205-251`` (per batch element).  ``one_pass`` streams
    the sampled keys once (``bsa_sampled_mass_onepass``): with 16 or 32
    samples and up to 473 blocks the per-row block log-sums stay on chip
    (TMEM and shared memory) and the kernel writes the mass itself; other
    shapes use a workspace and a reduction launch.  Otherwise every score is
    computed twice, once for the row's log-sum-exp and once for the
    normalised block sums (``bsa_sampled_mass``).
    """
    device = _require_cuda(q, k)
    if q.shape != k.shape or q.dim() != 4:
        raise ValueError("q and k must be [B, T, H, D] with equal shapes")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
        raise ValueError("sampled_block_mass expects bf16 inputs")
    if not 0 < samples <= block:
        raise ValueError("route_samples must be in [1, block_size]")
    if samples not in (1, 2, 4, 8, 16, 32):
        raise NotImplementedError("route_samples must be a power of two <= 32 on this path")
    B, T, H, D = q.shape
    if D != HEAD_DIM:
        raise NotImplementedError(f"head_dim must be {HEAD_DIM}")
    blocks = math.ceil(T / block)
    ids, bias = _device_sample_tables(T, block, samples, device)
    sq, sk = reorder_rows([q, k], ids)
    mass = torch.empty((B, H, blocks, blocks), dtype=torch.float32, device=device)
    s = float(scale) if scale is not None else D ** -0.5
    if one_pass and B * H <= 65535:
        lib = _native.load_library()
        nbytes = int(lib.bsa_sampled_mass_workspace_bytes(B, H, blocks, samples))
        work = (torch.empty((nbytes + 3) // 4, dtype=torch.float32, device=device)
                if nbytes else None)
        _native.call("bsa_sampled_mass_onepass", sq.data_ptr(), sk.data_ptr(), B, H, blocks,
                     samples, D, bias.data_ptr(), s, 1 if round_bf16 else 0,
                     work.data_ptr() if work is not None else None, nbytes, mass.data_ptr(),
                     _native.err_word(device).data_ptr(), _stream(device))
        return mass
    _native.call("bsa_sampled_mass", sq.data_ptr(), sk.data_ptr(), B, H, blocks, samples, D,
                 bias.data_ptr(), s, 1 if round_bf16 else 0, mass.data_ptr(),
                 _native.err_word(device).data_ptr(), _stream(device))
    return mass


def exact_block_mass(q: torch.Tensor, k: torch.Tensor, block: int = 128,
                     scale: float | None = None, lse: torch.Tensor | None = None) -> torch.Tensor:
    """Exact dense block mass ``[B, H, Qb, Qb]`` (reference ``flex.py:97-108,167-202``).

    ``lse``: fp32 ``[B, H, T]`` natural-log log-sum-exp of each query row (the
    dense pass's, as the reference passes it); without it the kernel computes
    it in a first pass.
    """
    device = _require_cuda(q, k, lse)
    if q.shape != k.shape or q.dim() != 4:
        raise ValueError("q and k must be [B, T, H, D] with equal shapes")
    q = q.to(torch.bfloat16).contiguous()
    k = k.to(torch.bfloat16).contiguous()
    B, T, H, D = q.shape
    if D != HEAD_DIM:
        raise NotImplementedError(f"head_dim must be {HEAD_DIM}")
    blocks = math.ceil(T / block)
    if lse is not None:
        if tuple(lse.shape) != (B, H, T):
            raise ValueError(f"lse must be [B, H, T] = {(B, H, T)}")
        lse = lse.to(torch.float32).contiguous()
    mass = torch.empty((B, H, blocks, blocks), dtype=torch.float32, device=device)
    s = float(scale) if scale is not None else D ** -0.5
    _native.call("bsa_exact_block_mass", q.data_ptr(), k.data_ptr(), B, T, H, D, block, s,
                 _native.ptr(lse), mass.data_ptr(), _native.err_word(device).data_ptr(),
                 _stream(device))
    return mass


class RouteCSR(NamedTuple):
    route: torch.Tensor | None    # uint8 [..., Qb, Kb]
    counts: torch.Tensor | None   # int32 [..., Qb]
    indices: torch.Tensor | None  # int32 [..., Qb, Kb]
    kept: torch.Tensor | None     # int64 [prod(...)] selected blocks per leading index


def keep_cap(cols: int, keep: float) -> int:
    """``max(1, math.ceil(cols * keep))`` exactly as the reference (``flex.py:89``)."""
    return max(1, math.ceil(cols * keep))


def route_select(mass: torch.Tensor, prev: torch.Tensor | None = None, persistence: float = 0.0,
                 target: float = 0.9, keep: float = 0.625, sink_blocks: int = 0,
                 want_route: bool = True, want_csr: bool = True,
                 want_kept: bool = True) -> RouteCSR:
    """Prior + top-mass + sink + CSR from fp32 ``mass [..., Qb, Kb]``.

    Bit-identical to the reference's ``_top_mass_route`` (``flex.py:83-94``)
    with the prior of ``flex.py:535-541`` and the sink of ``flex.py:550-566``.
    """
    device = _require_cuda(mass, prev)
    if mass.dtype != torch.float32:
        raise ValueError("mass must be float32")
    if not 0 < keep <= 1:
        raise ValueError("keep must be in (0, 1]")
    if not 0 < target <= 1:
        raise ValueError("mass_target must be in (0, 1]")
    mass = mass.contiguous()
    cols = mass.shape[-1]
    rows = mass.numel() // cols if cols else 0
    group = mass.shape[-2] if mass.dim() >= 2 else 1
    prev_u8 = None
    if prev is not None and persistence:
        if prev.shape != mass.shape:
            raise ValueError("previous route and mass must have identical shapes")
        prev_u8 = prev.to(torch.uint8).contiguous()
    lead = mass.shape[:-1]
    route = torch.empty(mass.shape, dtype=torch.uint8, device=device) if want_route else None
    counts = torch.empty(lead, dtype=torch.int32, device=device) if want_csr else None
    indices = torch.empty(mass.shape, dtype=torch.int32, device=device) if want_csr else None
    kept = (torch.empty(max(1, rows // max(1, group)), dtype=torch.int64, device=device)
            if want_kept else None)
    if rows:
        _native.call("bsa_route_select", mass.data_ptr(), _native.ptr(prev_u8), rows, cols,
                     group, float(persistence), float(target), keep_cap(cols, keep),
                     int(sink_blocks), _native.ptr(route), _native.ptr(counts),
                     _native.ptr(indices), _native.ptr(kept), _stream(device))
    return RouteCSR(route, counts, indices, kept)


def pack_boolean_rows(route: torch.Tensor):
    """CSR of a boolean route: counts and ids (selected ascending, then the rest)."""
    device = _require_cuda(route)
    if route.dim() < 2:
        raise ValueError("route must be a boolean tensor with at least two axes")
    cols = route.shape[-1]
    r = route.to(torch.uint8).contiguous()
    counts = torch.empty(route.shape[:-1], dtype=torch.int32, device=device)
    indices = torch.empty(route.shape, dtype=torch.int32, device=device)
    rows = r.numel() // cols if cols else 0
    if rows:
        _native.call("bsa_pack_boolean_rows", r.data_ptr(), rows, cols, counts.data_ptr(),
                     indices.data_ptr(), _stream(device))
    return counts, indices


# ----------------------------------------------------------------------------
# (f4) attention prologue
# ----------------------------------------------------------------------------

def qkv_prologue(q_proj: torch.Tensor, k_proj: torch.Tensor, v_proj: torch.Tensor, heads: int,
                 norm_q_weight: torch.Tensor | None = None,
                 norm_k_weight: torch.Tensor | None = None, eps: float = 1e-6,
                 rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
                 perm: torch.Tensor | None = None, norm_q: bool = True, norm_k: bool = True):
    """RMSNorm(Q), RMSNorm(K), RoPE(Q, K) and the reorder, in one pass.

    ``*_proj``: bf16 ``[B, T, H*D]`` (the ``to_q``/``to_k``/``to_v`` outputs;
    rows may be strided).  Returns bf16 ``q, k, v`` ``[B, T, H, D]`` with row i
    taken from token ``perm[i]``.  Bit-identical to the reference's
    ``rms_norm`` + ``apply_rope`` CPU path (``svg_ops.py:82-92,193-204``)
    followed by ``index_select(1, perm)``.
    """
    device = _require_cuda(q_proj, k_proj, v_proj)
    if not (q_proj.shape == k_proj.shape == v_proj.shape) or q_proj.dim() != 3:
        raise ValueError("projections must be [B, T, H*D] with equal shapes")
    if any(t.dtype != torch.bfloat16 for t in (q_proj, k_proj, v_proj)):
        raise ValueError("qkv_prologue expects bf16 projections")
    B, T, C = q_proj.shape
    if C % heads:
        raise ValueError(f"{C} features do not split into {heads} heads")
    D = C // heads
    if not (q_proj.stride() == k_proj.stride() == v_proj.stride()) or q_proj.stride(-1) != 1:
        q_proj, k_proj, v_proj = q_proj.contiguous(), k_proj.contiguous(), v_proj.contiguous()

    def weight(w):
        if w is None:
            return None
        if w.numel() != C:
            raise ValueError("norm weights must have H*D elements")
        return w.to(device=device, dtype=torch.float32).contiguous()
    wq, wk = weight(norm_q_weight), weight(norm_k_weight)
    if (rope_cos is None) != (rope_sin is None):
        raise ValueError("rope_cos and rope_sin go together")
    if rope_cos is not None:
        if tuple(rope_cos.shape) != (T, D // 2) or tuple(rope_sin.shape) != (T, D // 2):
            raise ValueError(f"rope tables must be [T, D/2] = {(T, D // 2)}")
        rope_cos = rope_cos.to(device=device, dtype=torch.float32).contiguous()
        rope_sin = rope_sin.to(device=device, dtype=torch.float32).contiguous()
    if perm is not None:
        perm = perm.to(device=device, dtype=torch.int32).contiguous()
        if perm.numel() != T:
            raise ValueError("perm must have T entries")
    outs = [torch.empty((B, T, heads, D), dtype=torch.bfloat16, device=device) for _ in range(3)]
    if B * T:
        st = q_proj.stride()
        _native.call("bsa_qkv_prologue", q_proj.data_ptr(), k_proj.data_ptr(), v_proj.data_ptr(),
                     B, T, heads, D, st[0], st[1], 1 if norm_q else 0, 1 if norm_k else 0,
                     _native.ptr(wq), _native.ptr(wk), float(eps), _native.ptr(rope_cos),
                     _native.ptr(rope_sin), _native.ptr(perm), outs[0].data_ptr(),
                     outs[1].data_ptr(), outs[2].data_ptr(), _native.err_word(device).data_ptr(),
                     _stream(device))
    return tuple(outs)


# ----------------------------------------------------------------------------
# (f3) directional frontier update
# ----------------------------------------------------------------------------

def _square_planes(t: torch.Tensor, name: str) -> tuple[int, int]:
    if t.dim() < 2 or t.shape[-1] != t.shape[-2]:
        raise ValueError(f"{name} must be [..., blocks, blocks]")
    blocks = t.shape[-1]
    return (t.numel() // (blocks * blocks) if blocks else 0), blocks


def _neighbors_i32(neighbors: torch.Tensor, blocks: int, device) -> torch.Tensor:
    if tuple(neighbors.shape) != (blocks, 4):
        raise ValueError("neighbors must have shape [blocks, 4]")
    return neighbors.to(device=device, dtype=torch.int32).contiguous()


def frontier_mask(route: torch.Tensor, neighbors: torch.Tensor) -> torch.Tensor:
    """Bool frontier of a route ``[..., Kb, Kb]`` (``routing.py:10-43``):
    selected cells with an unselected valid spatial neighbour along Q or K."""
    device = _require_cuda(route)
    planes, blocks = _square_planes(route, "route")
    nb = _neighbors_i32(neighbors, blocks, device)
    r = route.to(torch.uint8).contiguous()
    out = torch.empty(route.shape, dtype=torch.uint8, device=device)
    if planes:
        _native.call("bsa_frontier_mask", r.data_ptr(), nb.data_ptr(), planes, blocks,
                     out.data_ptr(), _native.err_word(device).data_ptr(), _stream(device))
    return out.bool()


class DirectionalResult(NamedTuple):
    route: torch.Tensor         # bool [..., Kb, Kb], after the sink
    frontier: torch.Tensor      # bool, frontier of ``route``
    candidates: torch.Tensor    # bool, expansion candidates (not in previous)
    exploration: torch.Tensor   # bool, exploration cells
    dropped: torch.Tensor       # bool, previous & ~route (before the sink)
    added: torch.Tensor         # bool, route & ~previous (before the sink)
    counts: torch.Tensor        # int32 [..., Kb] CSR counts of ``route``
    indices: torch.Tensor       # int32 [..., Kb, Kb] CSR ids
    kept: torch.Tensor          # int64 [planes] selected cells per plane


EXPAND_Q, EXPAND_K, EXPAND_JOINT = 1, 2, 4


def directional_update(mass: torch.Tensor, previous: torch.Tensor, neighbors: torch.Tensor, *,
                       keep: float, persistence: float = 0.5, min_ratio: float = 0.0,
                       candidate_bonus: float = 0.0, budget_scale: float = 1.0,
                       exploration_fraction: float = 0.0, expand_q: bool = True,
                       expand_k: bool = True, expand_joint: bool = True,
                       previous_frontier: torch.Tensor | None = None,
                       sink_blocks: int = 0) -> DirectionalResult:
    """Directional frontier update of ``previous`` from fp32 ``mass`` (both
    ``[..., Kb, Kb]``), then the first-frame sink and the CSR.

    Bit-identical to the reference's ``directional_budget_update``
    (``routing.py:97-168``) followed by ``_add_first_frame_sink``
    (``flex.py:550-566``); same argument checks and messages.
    """
    device = _require_cuda(mass, previous, previous_frontier)
    if previous.shape != mass.shape:
        raise ValueError("previous route and mass must have identical shapes")
    planes, blocks = _square_planes(mass, "mass")
    if tuple(neighbors.shape) != (blocks, 4):
        raise ValueError("neighbors must have shape [blocks, 4]")
    if budget_scale <= 0:
        raise ValueError("budget_scale must be positive")
    if not 0 <= exploration_fraction <= 1:
        raise ValueError("exploration_fraction must be in [0, 1]")
    if mass.dtype != torch.float32:
        raise ValueError("mass must be float32")
    if previous_frontier is not None and previous_frontier.shape != mass.shape:
        raise ValueError("previous_frontier and mass must have identical shapes")
    mass = mass.contiguous()
    prev = previous.to(torch.uint8).contiguous()
    front = previous_frontier.to(torch.uint8).contiguous() if previous_frontier is not None else None
    nb = _neighbors_i32(neighbors, blocks, device)
    explore = max(1, math.ceil(blocks * exploration_fraction)) if exploration_fraction else 0
    expand = ((EXPAND_Q if expand_q else 0) | (EXPAND_K if expand_k else 0)
              | (EXPAND_JOINT if expand_joint else 0))
    masks = torch.empty((6,) + tuple(mass.shape), dtype=torch.uint8, device=device)
    route, frontier, cand, expl, dropped, added = masks.unbind(0)
    counts = torch.empty(mass.shape[:-1], dtype=torch.int32, device=device)
    indices = torch.empty(mass.shape, dtype=torch.int32, device=device)
    kept = torch.empty(max(1, planes), dtype=torch.int64, device=device)
    if planes:
        _native.call("bsa_directional_update", mass.data_ptr(), prev.data_ptr(), nb.data_ptr(),
                     _native.ptr(front), planes, blocks, float(persistence), float(min_ratio),
                     float(candidate_bonus), float(budget_scale), keep_cap(blocks, keep), explore,
                     expand, int(sink_blocks), blocks, route.data_ptr(), frontier.data_ptr(),
                     cand.data_ptr(), expl.data_ptr(), dropped.data_ptr(), added.data_ptr(),
                     counts.data_ptr(), indices.data_ptr(), kept.data_ptr(),
                     _native.err_word(device).data_ptr(), _stream(device))
    else:
        kept.zero_()
    b = masks.bool()
    return DirectionalResult(b[0], b[1], b[2], b[3], b[4], b[5], counts, indices, kept[:planes])


# ----------------------------------------------------------------------------
# (a) attention
# ----------------------------------------------------------------------------

def dense_attention_block_mass(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                               scale: float | None = None,
                               workspace_bytes: int = 2 << 30):
    """Dense attention, its LSE and its exact block mass in one attention pass.

    ``q, k, v``: bf16 ``[B, T, H, 128]``.  Returns ``out`` bf16 ``[B, T, H, D]``,
    ``lse`` fp32 ``[B, H, T]`` (natural log) and ``mass`` fp32 ``[B, H, Qb, Qb]``
    over 128-token blocks: the reference's dense bootstrap (``flex.py:254-272``:
    FlexAttention with ``return_lse`` then ``_block_attention_mass``) without
    the second pass over the keys.  Heads go in chunks whose per-row block
    sums fit ``workspace_bytes``.
    """
    device = _require_cuda(q, k, v)
    if not (q.shape == k.shape == v.shape) or q.dim() != 4:
        raise ValueError("q, k and v must be [B, T, H, D] with equal shapes")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("dense_attention_block_mass expects bf16 q, k, v")
    B, T, H, D = q.shape
    if D != HEAD_DIM:
        raise NotImplementedError(f"head_dim must be {HEAD_DIM}")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    blocks = math.ceil(T / 128)
    out = torch.empty_like(q)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=device)
    mass = torch.empty((B, H, blocks, blocks), dtype=torch.float32, device=device)
    per_head = blocks * T * 4
    hc = max(1, min(H, workspace_bytes // per_head))
    work = torch.empty((hc, blocks, T), dtype=torch.float32, device=device)
    s = float(scale) if scale is not None else D ** -0.5
    st, ost = q.stride(), out.stride()
    esz = q.element_size()
    for b in range(B):
        for h0 in range(0, H, hc):
            n = min(hc, H - h0)
            off = (b * st[0] + h0 * st[2]) * esz
            ooff = (b * ost[0] + h0 * ost[2]) * esz
            _native.call("bsa_attention_dense_block_mass", q.data_ptr() + off,
                         k.data_ptr() + off, v.data_ptr() + off, 1, T, n, D, st[0], st[1], st[2],
                         s, out.data_ptr() + ooff, ost[0], ost[1], ost[2],
                         lse[b, h0:h0 + n].data_ptr(), work.data_ptr(),
                         mass[b, h0:h0 + n].data_ptr(), _native.err_word(device).data_ptr(),
                         _stream(device))
    return out, lse, mass


def block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           counts: torch.Tensor, indices: torch.Tensor, block: int = 128,
                           scale: float | None = None, out: torch.Tensor | None = None,
                           return_lse: bool = False, out_rows: torch.Tensor | None = None):
    """Block-sparse attention over a CSR route.

    ``q, k, v``: bf16 ``[B, T, H, D]``.  ``counts``: int32 ``[H, Qb]`` (one route
    for every batch element) or ``[B, H, Qb]``; ``indices``: int32 with a trailing
    ``route_cols >= Qb`` axis.  Returns bf16 ``[B, T, H, D]`` (and fp32 LSE
    ``[B, H, T]`` when ``return_lse``).  Reference ``flex.py:358-399``.
    ``out_rows`` (int32 ``[T]`` permutation on q's device): row i is written to
    token ``out_rows[i]`` of the output (``bsa_attention_fwd_scatter``), e.g. the
    spatial layout's pack permutation to get the output back in raster order
    without an unpack pass; the LSE stays in q's row order.
    """
    device = _require_cuda(q, k, v, counts, indices)
    if not (q.shape == k.shape == v.shape) or q.dim() != 4:
        raise ValueError("q, k and v must be [B, T, H, D] with equal shapes")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("block_sparse_attention expects bf16 q, k, v")
    B, T, H, D = q.shape
    if D != HEAD_DIM:
        raise NotImplementedError(f"head_dim must be {HEAD_DIM}")
    if block not in (64, 128):
        raise NotImplementedError("block must be 64 or 128")
    blocks = math.ceil(T / block)
    if counts.dim() == 2:
        has_batch = 0
        expect = (H, blocks)
    else:
        has_batch = 1
        expect = (B, H, blocks)
    if tuple(counts.shape) != expect:
        raise ValueError(f"counts shape {tuple(counts.shape)} != {expect}")
    if tuple(indices.shape[:-1]) != expect or indices.shape[-1] < blocks:
        raise ValueError("indices must be [..., Qb, route_cols >= Qb] matching counts")
    if counts.dtype != torch.int32 or indices.dtype != torch.int32:
        raise ValueError("counts and indices must be int32")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    counts = counts.contiguous()
    indices = indices.contiguous()
    if out is None:
        out = torch.empty_like(q)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=device) if return_lse else None
    s = float(scale) if scale is not None else D ** -0.5
    ost = out.stride()
    if out_rows is not None:
        if (out_rows.dtype != torch.int32 or out_rows.shape != (T,)
                or out_rows.device != q.device):
            raise ValueError("out_rows must be int32 [T] on q's device")
        out_rows = out_rows.contiguous()
        _native.call("bsa_attention_fwd_scatter", q.data_ptr(), k.data_ptr(), v.data_ptr(), B,
                     T, H, D, q.stride(0), q.stride(1), q.stride(2), counts.data_ptr(),
                     indices.data_ptr(), indices.shape[-1], has_batch, block, s,
                     out_rows.data_ptr(), out.data_ptr(), ost[0], ost[1], ost[2],
                     _native.ptr(lse), _native.err_word(device).data_ptr(), _stream(device))
        return (out, lse) if return_lse else out
    _native.call("bsa_attention_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), B, T, H, D,
                 q.stride(0), q.stride(1), q.stride(2), counts.data_ptr(), indices.data_ptr(),
                 indices.shape[-1], has_batch, block, s, out.data_ptr(), ost[0], ost[1], ost[2],
                 _native.ptr(lse), _native.err_word(device).data_ptr(), _stream(device))
    return (out, lse) if return_lse else out



def block_sparse_attention_peers(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                 counts: torch.Tensor, indices: torch.Tensor,
                                 peers: "PeerRows", block: int = 128,
                                 scale: float | None = None,
                                 out_rows: torch.Tensor | None = None) -> None:
    """Block-sparse attention of one branch (``[1, T, H, D]``) whose output
    rows go straight to the ranks holding their tokens (``bsa_attention_fwd_peers``):
    token ``t = out_rows[i]`` of packed row i lands in rank ``t // peers.tokens``'s
    buffer ``peers.ptrs[d]`` (strides ``peers.stride_t``, ``peers.stride_h``
    elements, this call's head h at ``h * stride_h``).  ``counts [H, Qb]``,
    ``indices [H, Qb, >= Qb]`` int32."""
    device = _require_cuda(q, k, v, counts, indices)
    if not (q.shape == k.shape == v.shape) or q.dim() != 4 or q.shape[0] != 1:
        raise ValueError("q, k and v must be [1, T, H, D] with equal shapes")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("block_sparse_attention_peers expects bf16 q, k, v")
    _, T, H, D = q.shape
    if D != HEAD_DIM:
        raise NotImplementedError(f"head_dim must be {HEAD_DIM}")
    blocks = math.ceil(T / block)
    if tuple(counts.shape) != (H, blocks) or tuple(indices.shape[:-1]) != (H, blocks):
        raise ValueError("counts must be [H, Qb] and indices [H, Qb, route_cols]")
    if counts.dtype != torch.int32 or indices.dtype != torch.int32:
        raise ValueError("counts and indices must be int32")
    if out_rows is not None and (out_rows.dtype != torch.int32 or out_rows.shape != (T,)
                                 or out_rows.device != q.device):
        raise ValueError("out_rows must be int32 [T] on q's device")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    counts, indices = counts.contiguous(), indices.contiguous()
    arr = (ctypes.c_void_p * len(peers.ptrs))(*peers.ptrs)
    s = float(scale) if scale is not None else D ** -0.5
    _native.call("bsa_attention_fwd_peers", q.data_ptr(), k.data_ptr(), v.data_ptr(), T, H, D,
                 q.stride(1), q.stride(2), counts.data_ptr(), indices.data_ptr(),
                 indices.shape[-1], block, s, _native.ptr(out_rows), arr, len(peers.ptrs),
                 peers.tokens, peers.stride_t, peers.stride_h,
                 _native.err_word(device).data_ptr(), _stream(device))


class PeerRows:
    """Destinations of a head-parallel output: ``ptrs[d]`` is rank d's output
    shard (mapped into this process), at this call's first head; ``tokens``
    tokens per rank; element strides ``stride_t``, ``stride_h``."""

    def __init__(self, ptrs, tokens, stride_t, stride_h):
        self.ptrs = [int(p) for p in ptrs]
        self.tokens = int(tokens)
        self.stride_t = int(stride_t)
        self.stride_h = int(stride_h)

    def shifted(self, heads: int, elem_bytes: int = 2) -> "PeerRows":
        """The same destinations ``heads`` heads further on."""
        off = heads * self.stride_h * elem_bytes
        return PeerRows([p + off for p in self.ptrs], self.tokens, self.stride_t, self.stride_h)


def ipc_export(t: torch.Tensor):
    """(64-byte CUDA IPC handle of ``t``'s allocation, ``t``'s byte offset in it)."""
    _require_cuda(t)
    handle = ctypes.create_string_buffer(64)
    offset = ctypes.c_int64(0)
    _native.call("bsa_ipc_export", t.data_ptr(), handle, ctypes.byref(offset))
    return bytes(handle.raw), int(offset.value)


def ipc_import(handle: bytes, offset: int) -> int:
    """Map another process's allocation on the current device; returns the
    device pointer at ``offset``."""
    if len(handle) != 64:
        raise ValueError("an IPC handle is 64 bytes")
    buf = ctypes.create_string_buffer(handle, 64)
    out = ctypes.c_void_p(0)
    _native.call("bsa_ipc_import", buf, int(offset), ctypes.byref(out))
    return int(out.value)


def ipc_release(ptr: int, offset: int) -> None:
    _native.call("bsa_ipc_release", int(ptr), int(offset))


def pull_rows(peer_shards: Sequence[int], peer_tokens: int, src_row_bytes: int,
              src_tensor_bytes: int, src_offset: int, dst: Sequence[torch.Tensor],
              perm: torch.Tensor | None = None) -> None:
    """Pull the packed rows of this call's heads from the ranks' input shards
    (``bsa_pull_rows``): ``dst[x][0, i]`` (``x`` = Q, K, V; ``[1, T, h, D]``
    contiguous) = ``row_bytes`` bytes of token ``t = perm[i]`` from rank
    ``t // peer_tokens``'s shard ``peer_shards[p]`` (device pointers)."""
    device = _require_cuda(*dst)
    if len(dst) != 3 or any(not d.is_contiguous() for d in dst):
        raise ValueError("dst must be three contiguous tensors")
    T = dst[0].shape[1]
    row_bytes = dst[0][0, 0].numel() * dst[0].element_size()
    if perm is not None and (perm.dtype != torch.int32 or perm.shape != (T,)
                             or perm.device != device):
        raise ValueError("perm must be int32 [T] on dst's device")
    arr = (ctypes.c_void_p * len(peer_shards))(*[int(p) for p in peer_shards])
    outs = (ctypes.c_void_p * 3)(*[d.data_ptr() for d in dst])
    _native.call("bsa_pull_rows", arr, len(peer_shards), int(peer_tokens), int(src_row_bytes),
                 int(src_tensor_bytes), int(src_offset), _native.ptr(perm), T, row_bytes, outs,
                 _native.err_word(device).data_ptr(), _stream(device))
