"""Build the in-tree CUDA library ``lib/libmoe_b200.so`` for sm_100a with nvcc.

Usage: python moe-680m_b200/build.py [--force] [--verbose]
Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (parallel), then linked into a
shared library with the CUDA runtime linked statically.  Rebuilds only when a source, header
or this script is newer than the library.
"""
from __future__ import annotations

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
LIB = PKG / "lib" / "libmoe_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-I", str(ROOT / "include")]


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return list(CSRC.glob("*")) + [ROOT / "include" / "moe_b200.h", Path(__file__)]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False,
          defines: tuple = (), out: Path | None = None) -> Path:
    """Compile the library; ``defines``/``out`` produce a variant elsewhere (e.g. a debug build
    with -DMOE_TC_TRACE) without touching the default library."""
    lib = Path(out) if out else LIB
    bdir = BUILD if not defines else BUILD.parent / ("_build_" + "_".join(d.lower() for d in defines))
    if not force and not defines and not needs_build():
        return LIB
    bdir.mkdir(exist_ok=True)
    lib.parent.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    extra = (["-Xptxas", "-v"] if ptxas_v else []) + [f"-D{d}" for d in defines]

    def compile_one(src: Path):
        obj = bdir / (src.stem + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, obj, cmd, r

    objs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for src, obj, cmd, r in ex.map(compile_one, srcs):
            if verbose or r.returncode != 0 or ptxas_v:
                sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}")
            objs.append(str(obj))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *objs, "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError("link failed")
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("--define", action="append", default=[], help="extra -D for a variant build")
    ap.add_argument("--out", default=None, help="output path of a variant build")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_v=a.ptxas_v, defines=tuple(a.define), out=a.out))
