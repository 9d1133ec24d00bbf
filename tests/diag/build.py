"""Build ``tests/diag/libbsa_diag.so`` (test-only diagnostics) for sm_100a.

It compiles ``diag.cu`` against the package's device helpers
(``dit_sparse_atten_b200/csrc/bsa_common.cuh``) with the same flags as
``libbsa.so``; rebuilt only when a source is newer.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
CSRC = REPO / "dit_sparse_atten_b200" / "csrc"
SOURCE = HERE / "diag.cu"
LIBRARY = HERE / "libbsa_diag.so"


def build(force: bool = False) -> Path:
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    from dit_sparse_atten_b200.csrc.build import NVCC_FLAGS, nvcc_path

    deps = [SOURCE, *CSRC.glob("*.cuh")]
    if (not force and LIBRARY.exists()
            and all(p.stat().st_mtime <= LIBRARY.stat().st_mtime for p in deps)):
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    subprocess.run([nvcc_path(), *NVCC_FLAGS, "-I", str(CSRC), "-shared", str(SOURCE),
                    "-o", str(tmp)], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force=True))
