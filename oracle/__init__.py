"""CPU oracle for the routed block-sparse attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``dit_sparse_atten_b200`` imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may use it, and only as the checker or
as the timed CPU baseline.

The oracle restates, in numpy, the arithmetic of the reference study
(yangshuo1230/DiT_Sparse_Atten, ``attention_backends/``) for the three parts of
the hot path:

* ``oracle.route``     sampled block mass, persistence prior, top-mass selection,
                       first-frame sink and the stable CSR pack
                       (``flex.py:83-94,205-251,535-566``; ``layout_ops.py:128-151``)
* ``oracle.attention`` block-sparse masked-softmax attention
                       (``sparse.py:670-751``; ``flex.py:379-399``)
* ``oracle.layout``    Morton microtile permutation and the sparse backend's
                       tile-major permutation (``spatial.py:19-183``;
                       ``sparse.py:51-138``)
* ``oracle.prologue``  the processor's Q/K RMSNorm, RoPE and the reorder
                       (``wan_diffusers.py:44-56``; ``svg_ops.py:82-92,193-204``)

Pinning: every function is checked against fixtures produced by importing the
reference itself (``tests/golden/make_golden.py``); see
``tests/test_oracle_golden.py``.
"""

from . import attention, layout, prologue, route, torch_cpu_order  # noqa: F401
