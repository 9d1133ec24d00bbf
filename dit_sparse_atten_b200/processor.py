"""Wan self-attention processor with the fused attention prologue.

Mirrors ``StudyWanProcessor`` of the reference (``wan_diffusers.py:21-70``):
same constructor ``(backend, layer_id)`` and call signature, installed with
``block.attn1.set_processor(...)`` (``wan_diffusers.py:208-210``).  The
difference is the prologue.  The Q/K RMSNorm, the head split, RoPE and,
when the backend packs its inputs, the spatial reorder run as one kernel
(``prologue.qkv_prologue``), and the backend is told that its inputs are
already packed (``packed_layout=``).  The projections (``to_q``, ``to_k``,
``to_v``, ``to_out``) stay the attention module's own layers.
"""

from __future__ import annotations

import torch

from . import prologue
from .context import set_routing_context


class StudyWanProcessor:
    """Attention processor for one Wan block's self-attention (``attn1``)."""

    def __init__(self, backend, layer_id):
        self.backend = backend
        self.layer_id = layer_id

    def __call__(self, attn, hidden_states, encoder_hidden_states=None, attention_mask=None,
                 rotary_emb=None, timestep=None):
        del timestep
        if encoder_hidden_states is not None:
            raise ValueError("StudyWanProcessor is only valid for Wan self-attention")
        set_routing_context(attention_id=self.layer_id)
        query = attn.to_q(hidden_states)
        key = attn.to_k(hidden_states)
        value = attn.to_v(hidden_states)
        if not (query.is_cuda and query.dtype == torch.bfloat16):
            raise RuntimeError("the fused attention prologue runs on CUDA bf16 projections only")
        finder = getattr(self.backend, "packed_layout_for", None)
        layout = finder(query.shape[1]) if finder is not None else None
        q, k, v = prologue.qkv_prologue(attn, query, key, value, rotary_emb, layout)
        extra = {"packed_layout": layout} if layout is not None else {}
        output = self.backend(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False,
                              window_size=(-1, -1), dtype=q.dtype,
                              attention_mask=attention_mask, **extra)
        output = output.flatten(2, 3).type_as(query)
        output = attn.to_out[0](output)
        output = attn.to_out[1](output)
        return output
