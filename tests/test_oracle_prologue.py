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
