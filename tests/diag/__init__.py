"""Test-only diagnostic kernels (``libbsa_diag.so``, built from ``diag.cu`` by
``build.py``): the softmax kernels' two exponential paths and one bounded
mbarrier wait that is made to time out.  Nothing in the package loads this
library."""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

from .build import LIBRARY, build

_lib = None


def load():
    global _lib
    if _lib is None:
        path = build()
        lib = ctypes.CDLL(str(path))
        lib.bsa_diag_exp2.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                      ctypes.c_int32, ctypes.c_void_p]
        lib.bsa_diag_exp2.restype = ctypes.c_int32
        lib.bsa_diag_unarmed_wait.argtypes = [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p]
        lib.bsa_diag_unarmed_wait.restype = ctypes.c_int32
        _lib = lib
    return _lib


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


def exp2(x: torch.Tensor, mode: str = "poly") -> torch.Tensor:
    """2^x through the softmax kernels' MUFU (``mode="mufu"``) or polynomial path."""
    x = x.to(torch.float32).contiguous()
    y = torch.empty_like(x)
    rc = load().bsa_diag_exp2(x.data_ptr(), y.data_ptr(), x.numel(),
                              1 if mode == "poly" else 0, _stream(x.device))
    if rc != 0:
        raise RuntimeError(f"bsa_diag_exp2 failed ({rc})")
    return y


def unarmed_wait(timeout_ns: int, err_word: torch.Tensor):
    """Run one bounded wait on a barrier nobody arrives on; returns the device
    result ``(completed, elapsed_ns, abort_flag)`` after synchronising."""
    result = torch.full((3,), -1, dtype=torch.int64, device=err_word.device)
    rc = load().bsa_diag_unarmed_wait(int(timeout_ns), err_word.data_ptr(), result.data_ptr(),
                                      _stream(err_word.device))
    if rc != 0:
        raise RuntimeError(f"bsa_diag_unarmed_wait failed ({rc})")
    torch.cuda.synchronize(err_word.device)
    return tuple(int(x) for x in result.cpu())
