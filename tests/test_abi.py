"""The C ABI library loads, exports every declared symbol, and validates arguments.

No call here reaches a kernel: each one fails argument validation first, so the
suite runs without a GPU.
"""

import ctypes
import re
from pathlib import Path

import pytest

from dit_sparse_atten_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "bsa.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"BSA_API\s+[\w\s\*]+?\b(bsa_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"bsa_version", "bsa_last_error", "bsa_reorder_rows", "bsa_pack_boolean_rows",
            "bsa_route_select", "bsa_sampled_mass", "bsa_exact_block_mass",
            "bsa_attention_fwd"} <= set(names)


def test_library_exports_every_declared_symbol():
    lib = _native.load_library()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _native.SIGNATURES, name
    assert lib.bsa_version() == 10000


def test_binding_arity_matches_header():
    text = HEADER.read_text()
    for name, (args, _res) in _native.SIGNATURES.items():
        m = re.search(r"\b" + name + r"\s*\(([^)]*)\)", text)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), name


def _err():
    return _native.load_library().bsa_last_error().decode()


def test_reorder_validates():
    lib = _native.load_library()
    assert lib.bsa_reorder_rows(0, None, None, None, 1, 1, 1, 16, None, None) == -1
    assert "n_tensors" in _err()
    src = (ctypes.c_void_p * 3)(0, 0, 0)
    assert lib.bsa_reorder_rows(1, src, src, 1, 1, 1, 1, 16, None, None) == -1
    assert "null" in _err()


def test_route_select_validates():
    lib = _native.load_library()
    assert lib.bsa_route_select(None, None, 1, 4, 1, 0.0, 0.9, 2, 0, None, None, None, None,
                                None) == -1
    assert lib.bsa_route_select(8, None, 1, 5000, 1, 0.0, 0.9, 2, 0, None, None, None, None,
                                None) == -2
    assert "4096" in _err()
    assert lib.bsa_route_select(8, None, 1, 4, 1, 0.0, 1.5, 2, 0, None, None, None, None,
                                None) == -1
    assert "mass_target" in _err()
    assert lib.bsa_route_select(8, None, 1, 4, 1, 0.0, 0.9, 0, 0, None, None, None, None,
                                None) == -1
    assert "max_blocks" in _err()
    assert lib.bsa_route_select(8, None, 3, 4, 2, 0.0, 0.9, 2, 0, None, None, None, 8,
                                None) == -1
    assert "rows_per_group" in _err()


def test_attention_and_mass_validate():
    lib = _native.load_library()
    args = (16, 16, 16, 1, 128, 4, 64, 16, 8, 16, 16, 2, 1, 0, 128, 0.1, 16, 1, 1, 1, None, None,
            None)
    assert lib.bsa_attention_fwd(*args) == -1  # null err_word
    args = (16, 16, 16, 1, 128, 4, 64, 16, 8, 16, 16, 2, 1, 0, 128, 0.1, 16, 1, 1, 1, None, 16,
            None)
    assert lib.bsa_attention_fwd(*args) == -2
    assert "head_dim" in _err()
    assert lib.bsa_sampled_mass(16, 16, 1, 1, 4, 3, 128, 16, 0.1, 1, 16, 16, None) == -2
    assert "samples" in _err()
    # one pass: 16 or 32 samples and up to 473 blocks need no workspace; past
    # that 2 x 40 x rows x (blocks + 1) floats, and a short workspace is refused
    assert lib.bsa_sampled_mass_workspace_bytes(2, 40, 450, 16) == 0
    assert lib.bsa_sampled_mass_workspace_bytes(2, 40, 473, 32) == 0
    assert lib.bsa_sampled_mass_workspace_bytes(2, 40, 474, 16) == 2 * 40 * 7584 * 475 * 4
    assert lib.bsa_sampled_mass_workspace_bytes(2, 40, 450, 8) == 2 * 40 * 3600 * 451 * 4
    assert lib.bsa_sampled_mass_onepass(16, 16, 2, 40, 474, 16, 128, 16, 0.1, 1, 16,
                                        2 * 40 * 7584 * 475 * 4 - 1, 16, 16, None) == -1
    assert "workspace" in _err()
    assert lib.bsa_exact_block_mass(16, 16, 1, 100, 1, 128, 96, 0.1, None, 16, 16, None) == -2
    assert "block" in _err()


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_native, "_lib", None)
    with pytest.raises(RuntimeError, match="missing"):
        _native.load_library(tmp_path / "libbsa.so")


def test_exchange_entry_points_validate():
    """The peer-memory exchange entry points refuse bad layouts before any
    device work: peer counts, token splits, alignment, rows that would read
    past a token's row or tensors that overlap."""
    lib = _native.load_library()
    err = ctypes.c_int32(0)
    peers = (ctypes.c_void_p * 8)(*([4096] * 8))
    dst = (ctypes.c_void_p * 3)(4096, 8192, 12288)
    ok_args = dict(n_peers=2, peer_tokens=8, src_row_bytes=256, src_tensor_bytes=8 * 256,
                   src_offset=0, tokens=16, row_bytes=128)

    def pull(**kw):
        a = {**ok_args, **kw}
        return lib.bsa_pull_rows(peers, a["n_peers"], a["peer_tokens"], a["src_row_bytes"],
                                 a["src_tensor_bytes"], a["src_offset"], None, a["tokens"],
                                 a["row_bytes"], dst, ctypes.byref(err), None)

    assert pull(n_peers=0) == -1 and "peers" in _err()
    assert pull(n_peers=9, tokens=72) == -1 and "peers" in _err()
    assert pull(tokens=15) == -1 and "tokens" in _err()
    assert pull(row_bytes=120) == -1 and "16-byte" in _err()
    assert pull(src_offset=160) == -1 and "inside a token's row" in _err()
    assert pull(src_tensor_bytes=7 * 256) == -1 and "overlap" in _err()
    assert lib.bsa_pull_rows(None, 2, 8, 256, 2048, 0, None, 16, 128, dst, ctypes.byref(err),
                             None) == -1 and "null" in _err()
    # attention with peer stores: peer count, token split, alignment, aliasing
    q = 65536

    def attn(out_peers, n, peer_tokens=8, tokens=16):
        return lib.bsa_attention_fwd_peers(q, q, q, tokens, 4, 128, 512, 128, 16, 16, 1, 128,
                                           0.1, None, out_peers, n, peer_tokens, 512, 128,
                                           ctypes.byref(err), None)

    out = (ctypes.c_void_p * 2)(4096, 8192)
    assert attn(out, 0) == -1 and "peers" in _err()
    assert attn(out, 9) == -1 and "peers" in _err()
    assert attn(out, 2, peer_tokens=7) == -1 and "tokens" in _err()
    assert attn((ctypes.c_void_p * 2)(4096, 8200), 2) == -1 and "aligned" in _err()
    assert attn((ctypes.c_void_p * 2)(4096, q), 2) == -1 and "alias" in _err()
