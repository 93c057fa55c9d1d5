"""Build the in-tree C-ABI shared library ``gdn_b200/libgdn_b200.so`` for sm_100a.

    python qwen-drive-edge-orin_b200/build.py [--force] [--verbose]

nvcc compiles ``csrc/*.cu`` with ``-gencode arch=compute_100a,code=sm_100a
-lineinfo -O3`` into one shared object (``-shared -Xcompiler -fPIC``), linked
only against the CUDA runtime. The library is rebuilt when any source or
header is newer than it. No GPU is needed to build.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT = PKG / "gdn_b200" / "libgdn_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources():
    return sorted(CSRC.glob("*.cu"))


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    deps.append(Path(__file__))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, extra=None) -> Path:
    if not force and not needs_build():
        return OUT
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xptxas", "-v" if verbose else "-O3", f"-I{INCLUDE}", f"-I{CSRC}",
           *(extra or []), *[str(s) for s in sources()], "-o", str(OUT) + ".tmp", "-cudart", "shared"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stdout.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
