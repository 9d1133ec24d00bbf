"""Build ``libbsa.so`` (the C ABI of include/bsa.h) for sm_100a with nvcc.

Usage: ``python -m dit_sparse_atten_b200.csrc.build [--verbose-ptxas]``.
The library is written next to the package (``dit_sparse_atten_b200/libbsa.so``)
so it travels with the source tree; it is rebuilt only when a source is newer.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PACKAGE = CSRC.parent
REPO = PACKAGE.parent
LIBRARY = PACKAGE / "libbsa.so"
SOURCES = sorted(CSRC.glob("*.cu"))
HEADERS = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [REPO / "include" / "bsa.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", str(REPO / "include"),
]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libbsa.so")


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in SOURCES + HEADERS if p.exists())


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    if not force and up_to_date():
        return LIBRARY
    nvcc = nvcc_path()
    objdir = REPO / "_build"
    objdir.mkdir(exist_ok=True)
    objects, commands = [], []
    for src in SOURCES:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose_ptxas:
            cmd[1:1] = ["-Xptxas", "-v"]
        commands.append(cmd)
        objects.append(str(obj))
    # one nvcc per translation unit, in parallel
    with ThreadPoolExecutor(max_workers=min(len(commands), os.cpu_count() or 1)) as pool:
        for done in pool.map(lambda c: subprocess.run(c, capture_output=True, text=True),
                             commands):
            sys.stdout.write(done.stdout)
            sys.stderr.write(done.stderr)
            done.check_returncode()
    tmp = LIBRARY.with_suffix(".so.tmp")
    subprocess.run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-o", str(tmp), *objects], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose-ptxas", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
