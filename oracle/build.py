"""Build the oracle's C restatements (test infrastructure; see oracle/__init__.py).

``python -m oracle.build`` compiles ``oracle/csrc/*.c`` with gcc into
``oracle/_build/liboracle.so``.  ``load()`` builds on first use.
"""

from __future__ import annotations

import ctypes
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCES = sorted((HERE / "csrc").glob("*.c"))
LIBRARY = HERE / "_build" / "liboracle.so"

_lib = None


def build(force: bool = False) -> Path:
    if not force and LIBRARY.exists() and all(
            s.stat().st_mtime <= LIBRARY.stat().st_mtime for s in SOURCES):
        return LIBRARY
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("a C compiler is needed to build the oracle")
    LIBRARY.parent.mkdir(exist_ok=True)
    tmp = LIBRARY.with_suffix(".tmp.so")
    subprocess.run([cc, "-O2", "-shared", "-fPIC", "-std=c99", "-o", str(tmp),
                    *map(str, SOURCES)], check=True)
    tmp.replace(LIBRARY)
    return LIBRARY


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        lib.oracle_argsort_desc.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_long,
                                            ctypes.c_void_p, ctypes.c_void_p]
        lib.oracle_argsort_desc.restype = None
        _lib = lib
    return _lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
