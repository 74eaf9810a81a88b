"""Build the in-tree CUDA library ``aeisu_b200/libaeisu_b200.so`` for sm_100a with nvcc.

    python -m aeisu_b200.build [--force] [--jobs N]

Objects go to ``aeisu_b200/_build/`` (git-ignored); the shared library sits in the package
directory so it travels with the source tree.  Rebuilds only when a source or header is
newer than the library.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libaeisu_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build aeisu_b200")
    return exe


def sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def headers():
    return sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h")))


def stale():
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources() + headers() + [Path(__file__)])


def compile_one(src: Path, verbose: bool):
    obj = BUILD / (src.name + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), *NVCC_FLAGS, "-x", "cu", *ARCH, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, (r.stdout + r.stderr).strip()


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: compile_one(s, verbose), srcs))
    for obj, log in results:
        if log and verbose:
            print(f"[{obj.name}]\n{log}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *[str(o) for o, _ in results], "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))


if __name__ == "__main__":
    sys.exit(main())
