"""Route bookkeeping on the device (``routing.py:10-41`` of the reference).

Only ``frontier_mask`` is provided: the non-directional sampled path records it
per state for ``profile_summary()``.  The directional budget update of the
reference (``routing.py:92-168``) is not part of this build.
"""

from __future__ import annotations

import torch


def _neighbor_values(tensor, neighbors, axis):
    heads, blocks, _ = tensor.shape
    values, valid_values = [], []
    for direction in range(neighbors.shape[1]):
        target = neighbors[:, direction].long()
        valid = target >= 0
        if axis == 1:
            idx = target.clamp_min(0).view(1, blocks, 1).expand(heads, blocks, blocks)
            gathered = torch.gather(tensor, 1, idx)
            valid_mask = valid.view(1, blocks, 1)
        else:
            idx = target.clamp_min(0).view(1, 1, blocks).expand(heads, blocks, blocks)
            gathered = torch.gather(tensor, 2, idx)
            valid_mask = valid.view(1, 1, blocks)
        values.append(gathered)
        valid_values.append(valid_mask.expand_as(tensor))
    return torch.stack(values, -1), torch.stack(valid_values, -1)


def frontier_mask(route, neighbors):
    """Selected route cells adjacent to an unselected spatial cell."""
    q_sel, q_valid = _neighbor_values(route, neighbors, axis=1)
    k_sel, k_valid = _neighbor_values(route, neighbors, axis=2)
    return (route & (q_valid & ~q_sel).any(-1)) | (route & (k_valid & ~k_sel).any(-1))
