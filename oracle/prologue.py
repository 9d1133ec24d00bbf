"""Attention prologue of the reference's Wan processor, restated in numpy
(test oracle; see ``oracle/__init__``).

``wan_diffusers.py:44-56``: ``rms_norm`` of the Q and K projections over the
flattened ``H*D`` features (``svg_ops.py:82-92``, the CPU path: float32
``x * rsqrt(mean(x^2) + eps) * weight``, stored in the input dtype), the head
split, ``apply_rope`` (``svg_ops.py:193-204``: pairs of channels as complex
numbers times the rotary table, in float64, stored in the input dtype), and
then the backend's spatial reorder (``spatial.py:86-93``).
"""

from __future__ import annotations

import numpy as np

from . import torch_cpu_order as order
from .route import round_bf16


def rms_norm(x, weight, eps):
    """bf16-valued ``[..., C]`` -> bf16-valued float32 (``svg_ops.py:84-92``)."""
    v = np.asarray(x, np.float32)
    ms = order.row_mean(np.square(v, dtype=np.float32))[..., None]
    out = (v * (np.float32(1.0) / np.sqrt(ms + np.float32(eps), dtype=np.float32))).astype(
        np.float32)
    if weight is not None:
        out = (out * np.asarray(weight, np.float32)).astype(np.float32)
    return round_bf16(out)


def apply_rope(x, cos, sin):
    """``x`` bf16-valued ``[B, T, H, D]``; ``cos``/``sin`` ``[T, D/2]`` (the real and
    imaginary parts of the rotary table): channel pairs (2j, 2j+1) rotate by
    angle j of their token (``svg_ops.py:199-204``)."""
    xd = np.asarray(x, np.float64)
    re, im = xd[..., 0::2], xd[..., 1::2]
    c = np.asarray(cos, np.float64)[None, :, None, :]
    s = np.asarray(sin, np.float64)[None, :, None, :]
    out = np.empty_like(xd)
    out[..., 0::2] = re * c - im * s
    out[..., 1::2] = re * s + im * c
    return round_bf16(out.astype(np.float32))


def qkv_prologue(q_proj, k_proj, v_proj, heads, norm_q_weight, norm_k_weight, eps, cos, sin,
                 perm=None):
    """``[B, T, H*D]`` projections -> ``q, k, v`` ``[B, T, H, D]`` in packed
    order ``out[:, i] = x[:, perm[i]]`` (identity without ``perm``)."""
    B, T, C = q_proj.shape
    D = C // heads
    q = rms_norm(q_proj, norm_q_weight, eps) if norm_q_weight is not False else np.asarray(
        q_proj, np.float32)
    k = rms_norm(k_proj, norm_k_weight, eps) if norm_k_weight is not False else np.asarray(
        k_proj, np.float32)
    q, k = q.reshape(B, T, heads, D), k.reshape(B, T, heads, D)
    v = np.asarray(v_proj, np.float32).reshape(B, T, heads, D)
    if cos is not None:
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
    if perm is not None:
        idx = np.asarray(perm, np.int64)
        q, k, v = q[:, idx], k[:, idx], v[:, idx]
    return q, k, v
