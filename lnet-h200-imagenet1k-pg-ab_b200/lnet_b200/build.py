"""Build the lnet_b200 CUDA library in-tree for sm_100a.

``build()`` compiles every ``csrc/*.cu`` with nvcc into
``lnet_b200/_lib/liblnet_b200.so`` (a C-ABI shared library loaded with
ctypes).  Rebuilds only when a source or header is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent  # the package directory holding csrc/
REPO = ROOT.parent
CSRC = ROOT / "csrc"
INCLUDE = REPO / "include"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "liblnet_b200.so"
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the lnet_b200 CUDA library cannot be built")
    return cand


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = ROOT / "_build"
    obj_dir.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    flags = [
        "-O3", "-std=c++17", ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
        f"-I{INCLUDE}", f"-I{CSRC}",
    ]
    objs = []
    procs = []
    for src in _sources():
        obj = obj_dir / (src.stem + ".o")
        objs.append(obj)
        cmd = [nvcc, *flags, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    for cmd, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{out.decode()}")
        if verbose and out:
            print(out.decode())
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcublas"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose=True))
