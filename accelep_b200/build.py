"""Builds libaccelep_b200.so in-tree (accelep_b200/lib/) with nvcc for sm_100a.

    python -m accelep_b200.build [--verbose-ptxas]

Every CUDA and C++ source under accelep_b200/csrc is compiled to an object in
accelep_b200/_build and linked into one shared library with the CUDA runtime
linked statically, so the library does not depend on which libcudart another
library in the process (PyTorch's, for one) brought along.
"""

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libaccelep_b200.so"
INCLUDE = ROOT / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden,-Wall",
          f"-I{INCLUDE}", f"-I{CSRC}"]


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cc")))


def _compile(src, verbose_ptxas):
    obj = BUILD / (src.name + ".o")
    cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["--expt-relaxed-constexpr"]
        if verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{out.stdout}\n{out.stderr}")
    return obj, out.stderr


def _stale(objs):
    if not LIB.is_file():
        return True
    lib_time = LIB.stat().st_mtime
    headers = list(INCLUDE.glob("*.h")) + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh"))
    newest = max(p.stat().st_mtime for p in list(_sources()) + headers + [Path(__file__)])
    return newest > lib_time or any(not o.is_file() for o in objs)


def build(force=False, verbose_ptxas=False, quiet=True):
    """Compiles and links the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    objs = [BUILD / (s.name + ".o") for s in srcs]
    if not force and not _stale(objs):
        return LIB
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        for obj, log in pool.map(lambda s: _compile(s, verbose_ptxas), srcs):
            logs.append(log)
    link = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static",
            "-Xlinker", "-Bsymbolic", "-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"]
    out = subprocess.run(link, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"link failed: {' '.join(link)}\n{out.stdout}\n{out.stderr}")
    if verbose_ptxas or not quiet:
        sys.stderr.write("".join(logs))
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas, quiet=False))


if __name__ == "__main__":
    main()
