"""The prologue oracle (``oracle/prologue.py``) against the reference's own
``rms_norm`` + ``apply_rope`` CPU path and its layout reorder
(``tests/golden/prologue.npz``), bit for bit."""

import numpy as np
import torch

from conftest import sha256_tensor
from dit_sparse_atten_b200 import synthetic
from oracle import prologue as opro

CASE = {"batch": 1, "grid": (1, 8, 16), "heads": 2, "seed": 12, "eps": 1e-6}


def prologue_case():
    (qp, kp, vp), (wq, wk), rotary = synthetic.prologue_inputs(
        CASE["batch"], CASE["grid"], CASE["heads"], seed=CASE["seed"])
    return (qp, kp, vp), (wq, wk), rotary


def bf16_bits_to_float(bits):
    return (np.asarray(bits).astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_inputs_match_fixture_digests(golden):
    g = golden("prologue.npz")
    (qp, kp, vp), (wq, wk), rotary = prologue_case()
    assert [sha256_tensor(x) for x in (qp, kp, vp)] == list(g["proj_sha"])
    assert [sha256_tensor(w) for w in (wq, wk)] == list(g["weight_sha"])
    assert sha256_tensor(torch.view_as_real(rotary)) == str(g["rotary_sha"])


def test_oracle_matches_reference(golden):
    g = golden("prologue.npz")
    (qp, kp, vp), (wq, wk), rotary = prologue_case()
    q, k, v = opro.qkv_prologue(qp.float().numpy(), kp.float().numpy(), vp.float().numpy(),
                                CASE["heads"], wq.float().numpy(), wk.float().numpy(),
                                CASE["eps"], rotary.real.numpy(), rotary.imag.numpy(),
                                perm=g["perm"])
    for name, got in (("q", q), ("k", k), ("v", v)):
        assert np.array_equal(got, bf16_bits_to_float(g[name])), name


def test_rotation_products_are_exact_in_float64():
    """The CUDA rotation rounds re*c - im*s (and re*s + im*c) once, by a fused
    multiply-add on float64.  That equals the reference's float64 product
    then subtraction only if every product of a bf16 value (8 significant
    bits) and a float32 factor (24 bits) is exact in float64.  Checked here
    with exact rationals on seeded values across the exponent range, and the
    single rounding of the difference against the product-then-subtract."""
    from fractions import Fraction
    rng = np.random.default_rng(21)
    n = 4000
    x = (rng.standard_normal(n) * np.exp2(rng.integers(-40, 40, n))).astype(np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()          # bf16 values
    ang = rng.uniform(-np.pi, np.pi, n)
    c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    re, im = xb[: n // 2], xb[n // 2:]
    for a, b in ((re, c[: n // 2]), (im, s[n // 2:]), (re, s[: n // 2]), (im, c[n // 2:])):
        for u, w in zip(a.tolist(), b.tolist()):
            assert float(u) * float(w) == Fraction(u) * Fraction(w)
    cc, ss = c[: n // 2].astype(np.float64), s[: n // 2].astype(np.float64)
    for u, v, cv, sv in zip(re.tolist(), im.tolist(), cc.tolist(), ss.tolist()):
        # one rounding of the exact difference == rounding of exact products' difference
        exact = Fraction(u) * Fraction(cv) - Fraction(v) * Fraction(sv)
        assert float(exact) == u * cv - v * sv
