"""ctypes binding of ``libbsa.so`` (the C ABI declared in ``include/bsa.h``).

The library is required: every sparse-path operation raises ``RuntimeError``
when it is missing or when a call fails; there is no CPU substitute.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().with_name("libbsa.so")

# Entry points and their C signatures (include/bsa.h).
_I32, _I64, _F32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float
_P = ctypes.c_void_p
SIGNATURES = {
    "bsa_version": ([], _I32),
    "bsa_last_error": ([], ctypes.c_char_p),
    "bsa_reorder_rows": ([_I32, _P, _P, _P, _I64, _I64, _I64, _I64, _P, _P], _I32),
    "bsa_gather_scatter_rows": ([_I32, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P],
                                _I32),
    "bsa_pack_boolean_rows": ([_P, _I64, _I32, _P, _P, _P], _I32),
    "bsa_route_select": ([_P, _P, _I64, _I32, _I32, _F32, _F32, _I32, _I32, _P, _P, _P, _P, _P],
                         _I32),
    "bsa_qkv_prologue": ([_P, _P, _P, _I64, _I64, _I64, _I32, _I64, _I64, _I32, _I32, _P, _P,
                          _F32, _P, _P, _P, _P, _P, _P, _P, _P], _I32),
    "bsa_frontier_mask": ([_P, _P, _I64, _I32, _P, _P, _P], _I32),
    "bsa_directional_update": ([_P, _P, _P, _P, _I64, _I32, _F32, _F32, _F32, _F32, _I32, _I32,
                                _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
                               _I32),
    "bsa_sampled_mass": ([_P, _P, _I64, _I64, _I32, _I32, _I32, _P, _F32, _I32, _P, _P, _P], _I32),
    "bsa_sampled_mass_noalloc": ([_P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _F32, _I32, _P, _P,
                                  _P], _I32),
    "bsa_sampled_mass_workspace_bytes": ([_I64, _I64, _I32, _I32], _I64),
    "bsa_sampled_mass_onepass": ([_P, _P, _I64, _I64, _I32, _I32, _I32, _P, _F32, _I32, _P, _I64,
                                  _P, _P, _P], _I32),
    "bsa_exact_block_mass": ([_P, _P, _I64, _I64, _I64, _I32, _I32, _F32, _P, _P, _P, _P], _I32),
    "bsa_attention_fwd": ([_P, _P, _P, _I64, _I64, _I64, _I32, _I64, _I64, _I64, _P, _P, _I32,
                           _I32, _I32, _F32, _P, _I64, _I64, _I64, _P, _P, _P], _I32),
    "bsa_attention_fwd_scatter": ([_P, _P, _P, _I64, _I64, _I64, _I32, _I64, _I64, _I64, _P, _P,
                                   _I32, _I32, _I32, _F32, _P, _P, _I64, _I64, _I64, _P, _P, _P],
                                  _I32),
    "bsa_attention_dense_block_mass": ([_P, _P, _P, _I64, _I64, _I64, _I32, _I64, _I64, _I64,
                                        _F32, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P], _I32),
    "bsa_attention_fwd_peers": ([_P, _P, _P, _I64, _I64, _I32, _I64, _I64, _P, _P, _I32, _I32,
                                 _F32, _P, _P, _I32, _I64, _I64, _I64, _P, _P], _I32),
    "bsa_pull_rows": ([_P, _I32, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _P, _P], _I32),
    "bsa_ipc_export": ([_P, _P, ctypes.POINTER(ctypes.c_int64)], _I32),
    "bsa_ipc_import": ([_P, _I64, ctypes.POINTER(ctypes.c_void_p)], _I32),
    "bsa_ipc_release": ([_P, _I64], _I32),
}

DEVICE_ERRORS = {
    1: "a bounded wait inside a kernel timed out",
    2: "a route/permutation entry was out of range",
    4: "tensor-memory allocation failed",
    8: "the kernel's shared-memory layout did not fit",
}

_lock = threading.Lock()
_lib = None
_err_words: dict = {}


def load_library(path: Path | None = None) -> ctypes.CDLL:
    """Load ``libbsa.so`` once and bind every entry point's signature.

    The library next to this file is used unless ``path`` or the environment
    variable ``BSA_LIBRARY_PATH`` names another build.
    """
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if path is None and os.environ.get("BSA_LIBRARY_PATH"):
            path = os.environ["BSA_LIBRARY_PATH"]
        target = Path(path) if path is not None else LIBRARY_PATH
        if not target.exists():
            raise RuntimeError(
                f"{target} is missing: build it with `python -m dit_sparse_atten_b200.csrc.build` "
                "(the sparse attention path has no non-CUDA implementation)")
        lib = ctypes.CDLL(str(target))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Call an entry point; raise ``RuntimeError`` with its message on failure."""
    lib = load_library()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.bsa_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed ({rc}): {msg}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def err_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 error word the kernels OR their ``BSA_DEVICE_*`` bits into."""
    device = torch.device(device)
    key = device.index if device.index is not None else torch.cuda.current_device()
    word = _err_words.get(key)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=device)
        _err_words[key] = word
    return word


def check_device_errors(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronise on the error word and raise if any kernel reported a problem."""
    keys = list(_err_words) if device is None else [torch.device(device).index or 0]
    for key in keys:
        word = _err_words.get(key)
        if word is None:
            continue
        value = int(word.item())
        if value:
            if reset:
                word.zero_()
            reasons = [text for bit, text in DEVICE_ERRORS.items() if value & bit]
            raise RuntimeError(f"libbsa kernel error 0x{value:x}: " + "; ".join(reasons))
