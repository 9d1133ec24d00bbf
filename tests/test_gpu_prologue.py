"""GPU parity of the attention prologue (``csrc/prologue.cu``: RMSNorm of Q/K,
RoPE, reorder in one pass) through the C ABI, against the reference's
outputs (``tests/golden/prologue.npz``) and the oracle: bit-exact."""

import numpy as np
import pytest
import torch

from dit_sparse_atten_b200 import _native, kernels, synthetic
from dit_sparse_atten_b200.spatial import build_spatial_layout
from oracle import prologue as opro
from test_oracle_prologue import CASE, bf16_bits_to_float, prologue_case

pytestmark = pytest.mark.gpu
DEV = "cuda"


def run(proj, weights, rotary, heads, perm, eps=1e-6, norm=(True, True), rope=True):
    qp, kp, vp = (x.to(DEV) for x in proj)
    wq, wk = weights
    cos = rotary.real.float() if rope else None
    sin = rotary.imag.float() if rope else None
    out = kernels.qkv_prologue(qp, kp, vp, heads, wq, wk, eps, cos, sin,
                               perm=None if perm is None else torch.as_tensor(perm),
                               norm_q=norm[0], norm_k=norm[1])
    torch.cuda.synchronize()
    _native.check_device_errors()
    return [o.float().cpu().numpy() for o in out]


def oracle(proj, weights, rotary, heads, perm, eps=1e-6, norm=(True, True), rope=True):
    qp, kp, vp = (x.float().cpu().numpy() for x in proj)
    wq, wk = (None if w is None else w.float().numpy() for w in weights)
    return opro.qkv_prologue(qp, kp, vp, heads, wq if norm[0] else False,
                             wk if norm[1] else False, eps,
                             rotary.real.numpy() if rope else None,
                             rotary.imag.numpy() if rope else None, perm=perm)


def test_matches_reference_fixture(golden):
    g = golden("prologue.npz")
    proj, weights, rotary = prologue_case()
    got = run(proj, weights, rotary, CASE["heads"], g["perm"])
    for name, arr in zip("qkv", got):
        assert np.array_equal(arr, bf16_bits_to_float(g[name])), name


@pytest.mark.parametrize("batch,grid,heads,variant", [
    (2, (2, 5, 48), 40, "full"),       # Wan heads, 480 tokens, partial last block
    (1, (2, 8, 16), 3, "no_weight"),
    (1, (2, 8, 16), 3, "no_rope"),
    (2, (1, 8, 16), 2, "no_norm_k"),
    (1, (2, 8, 16), 2, "strided"),     # projections as column slices of one [B, T, 3C] tensor
])
def test_matches_oracle(batch, grid, heads, variant):
    proj, weights, rotary = synthetic.prologue_inputs(batch, grid, heads, seed=heads + batch)
    perm = build_spatial_layout(grid, 128).permutation_cpu.numpy()
    kw = {}
    if variant == "no_weight":
        weights = (None, None)
    if variant == "no_rope":
        kw["rope"] = False
    if variant == "no_norm_k":
        kw["norm"] = (True, False)
    if variant == "strided":
        fused = torch.cat(proj, -1)
        C = proj[0].shape[-1]
        proj = [fused[..., i * C:(i + 1) * C] for i in range(3)]
        assert proj[0].stride(1) == 3 * C
    got = run(proj, weights, rotary, heads, perm, **kw)
    ref = oracle(proj, weights, rotary, heads, perm, **kw)
    for name, a, r in zip("qkv", got, ref):
        assert np.array_equal(a, r), (name, int((a != r).sum()))


def test_identity_order_and_bad_perm_entry():
    proj, weights, rotary = synthetic.prologue_inputs(1, (1, 8, 16), 2, seed=3)
    got = run(proj, weights, rotary, 2, None)
    ref = oracle(proj, weights, rotary, 2, None)
    assert all(np.array_equal(a, r) for a, r in zip(got, ref))
    perm = torch.arange(128, dtype=torch.int32)
    perm[5] = 500
    kernels.qkv_prologue(*(x.to(DEV) for x in proj), 2, *weights, 1e-6, rotary.real.float(),
                         rotary.imag.float(), perm=perm)
    with pytest.raises(RuntimeError, match="out of range"):
        _native.check_device_errors()
