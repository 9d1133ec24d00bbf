"""The attention prologue of the reference's Wan processor on the GPU
(``wan_diffusers.py:44-56``): RMSNorm of the Q and K projections, the rotary
embedding, and the spatial reorder into route-block order, in one kernel
(``csrc/prologue.cu``) instead of the reference's five full-tensor passes
(two norms, the head transposes, RoPE, the backend's reorder).
"""

from __future__ import annotations

import torch

from . import kernels


def rope_tables(rotary_emb: torch.Tensor):
    """``(cos, sin)`` fp32 ``[T, D/2]`` of a complex rotary table shaped like the
    reference's ``rotary_emb`` (``[1, 1, T, D/2]`` or ``[T, D/2]``; the real and
    imaginary parts that ``svg_ops.apply_rope`` passes to its kernel)."""
    table = rotary_emb.reshape(rotary_emb.shape[-2], rotary_emb.shape[-1])
    return table.real.float().contiguous(), table.imag.float().contiguous()


def qkv_prologue(attn, query, key, value, rotary_emb=None, layout=None):
    """``query``/``key``/``value``: the ``to_q``/``to_k``/``to_v`` outputs
    ``[B, T, H*D]`` of a Wan attention module ``attn`` (``heads``, ``norm_q``,
    ``norm_k`` as in diffusers).  Returns ``[B, T, H, D]`` tensors, in the route
    -block order of ``layout`` (a ``SpatialTokenLayout``) when one is given."""
    norm_q, norm_k = getattr(attn, "norm_q", None), getattr(attn, "norm_k", None)
    eps = (norm_q.eps if norm_q is not None else norm_k.eps if norm_k is not None else 1e-6)
    if norm_q is not None and norm_k is not None and norm_q.eps != norm_k.eps:
        raise NotImplementedError("norm_q and norm_k with different eps")
    cos = sin = None
    if rotary_emb is not None:
        cos, sin = rope_tables(rotary_emb)
    perm = layout.permutation_cpu if layout is not None else None
    return kernels.qkv_prologue(
        query, key, value, attn.heads,
        norm_q_weight=getattr(norm_q, "weight", None), norm_k_weight=getattr(norm_k, "weight", None),
        eps=eps, rope_cos=cos, rope_sin=sin, perm=perm,
        norm_q=norm_q is not None, norm_k=norm_k is not None)
