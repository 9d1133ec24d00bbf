"""Exact float32 evaluation order of the reference's CPU reductions (test oracle).

The reference's top-mass rule (``attention_backends/flex.py:86-89``) compares a
float32 prefix sum against ``mass.sum(-1) * target``.  Which blocks are kept
depends on the last bit of both values, so the oracle (and the CUDA selection
kernel) must reproduce the order in which the reference's PyTorch CPU build
evaluates them.  The rules below were pinned empirically against torch 2.11 CPU
(``tests/golden/make_golden.py`` stores the reference's own outputs and
``tests/test_oracle_golden.py`` re-checks them bit for bit):

* ``Tensor.sum(-1)`` over a contiguous float32 row of length ``n``:
  ATen's cascade sum.  With ``W = 8`` float lanes and an ILP factor of 4, lane
  accumulator ``(k, lane)`` adds, in order, elements ``(4*i + k)*W + lane`` for
  ``i < n // (4W)``, using a 4-level cascade with level step ``2**max(4,
  ceil(log2(size)) // 4)``; the four ILP accumulators are folded into the first,
  then the scalar tail ``x[(n//W)*W:]`` is summed from 0 and the 8 lanes are
  added to it in lane order.  Rows shorter than ``W`` use the same scheme on
  scalars (4 accumulators).
* ``Tensor.cumsum(-1)``: sequential accumulation in float64, each prefix
  rounded to float32.
* ``Tensor.mean(-1)``: ``fl32(sum / n)`` with the sum above.
* ``Tensor * python_float``: ``fl32(x * fl32(scalar))``.
"""

from __future__ import annotations

import numpy as np

LANES = 8
ILP = 4
LEVELS = 4


def _ceil_log2(value: int) -> int:
    return 0 if value <= 1 else (value - 1).bit_length()


def _multi_row_sum(chunks: np.ndarray) -> np.ndarray:
    """Cascade-sum ``chunks[size, nrows, lanes]`` over axis 0 (ATen multi_row_sum).

    Vectorised over any leading batch axis placed after ``size``.
    """
    size = chunks.shape[0]
    level_power = max(4, _ceil_log2(size) // LEVELS)
    level_step = 1 << level_power
    level_mask = level_step - 1
    acc = np.zeros((LEVELS,) + chunks.shape[1:], np.float32)
    i = 0
    while i + level_step <= size:
        for _ in range(level_step):
            acc[0] = acc[0] + chunks[i]
            i += 1
        for j in range(1, LEVELS):
            acc[j] = acc[j] + acc[j - 1]
            acc[j - 1] = 0
            if (i & (level_mask << (j * level_power))) != 0:
                break
    while i < size:
        acc[0] = acc[0] + chunks[i]
        i += 1
    for j in range(1, LEVELS):
        acc[0] = acc[0] + acc[j]
    return acc[0]


def row_sum(x: np.ndarray) -> np.ndarray:
    """float32 ``x.sum(-1)`` in the reference's CPU evaluation order."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    n = x.shape[-1]
    rows = x.reshape(-1, n)
    if n < LANES:
        size_ilp = n // ILP
        chunks = rows[:, : size_ilp * ILP].reshape(rows.shape[0], size_ilp, ILP).transpose(1, 0, 2)
        partial = _multi_row_sum(chunks)  # [rows, ILP]
        p0 = partial[:, 0].copy()
        for i in range(size_ilp * ILP, n):
            p0 = p0 + rows[:, i]
        for k in range(1, ILP):
            p0 = p0 + partial[:, k]
        return (np.float32(0) + p0).astype(np.float32).reshape(lead)
    vec_size = n // LANES
    size_ilp = vec_size // ILP
    vecs = rows[:, : vec_size * LANES].reshape(rows.shape[0], vec_size, LANES)
    chunks = vecs[:, : size_ilp * ILP].reshape(rows.shape[0], size_ilp, ILP, LANES).transpose(1, 0, 2, 3)
    partial = _multi_row_sum(chunks)  # [rows, ILP, LANES]
    p0 = partial[:, 0].copy()
    for i in range(size_ilp * ILP, vec_size):
        p0 = p0 + vecs[:, i]
    for k in range(1, ILP):
        p0 = p0 + partial[:, k]
    final = np.zeros(rows.shape[0], np.float32)
    for i in range(vec_size * LANES, n):
        final = final + rows[:, i]
    for lane in range(LANES):
        final = final + p0[:, lane]
    return final.astype(np.float32).reshape(lead)


def row_mean(x: np.ndarray) -> np.ndarray:
    """float32 ``x.mean(-1)``: ``fl32(sum / n)``."""
    return (row_sum(x) / np.float32(x.shape[-1])).astype(np.float32)


def cumsum(x: np.ndarray) -> np.ndarray:
    """float32 ``x.cumsum(-1)``: float64 accumulation, rounded per prefix."""
    return np.cumsum(np.asarray(x, np.float64), axis=-1).astype(np.float32)


def mul_scalar(x: np.ndarray, scalar: float) -> np.ndarray:
    """float32 ``x * scalar`` for a Python float scalar."""
    return (np.asarray(x, np.float32) * np.float32(scalar)).astype(np.float32)
