"""Dense attention fallback (the reference's ``DenseBackend``, ``dense.py:14-48``).

Used exactly where the reference uses it: layer 0, step-0 dense output, routes
dispatched to dense, cross-attention and unsupported modes.  It calls the
library SDPA kernel.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


class DenseBackend:
    name = "dense"

    def __call__(self, q, k, v, q_lens=None, k_lens=None, dropout_p=0.0, softmax_scale=None,
                 q_scale=None, causal=False, window_size=(-1, -1), deterministic=False,
                 dtype=torch.bfloat16, version=None, **_):
        del q_lens, k_lens, deterministic, version
        if window_size != (-1, -1):
            raise NotImplementedError("The dense SDPA backend only supports global attention")
        output_dtype = q.dtype
        q = q.transpose(1, 2).to(dtype)
        k = k.transpose(1, 2).to(dtype)
        v = v.transpose(1, 2).to(dtype)
        if q_scale is not None:
            q = q * q_scale
        output = F.scaled_dot_product_attention(q, k, v, dropout_p=dropout_p, is_causal=causal,
                                                scale=softmax_scale)
        return output.transpose(1, 2).contiguous().to(output_dtype)
