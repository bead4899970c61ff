"""Builds libdak_b200.so (the C ABI in include/dak_b200.h) for sm_100a.

The library is compiled in-tree with nvcc, linked against the static CUDA
runtime, and loaded by `directaccesskernel_b200._lib` through ctypes.  It needs
no torch headers.  Usage: ``python -m directaccesskernel_b200.build [--verbose]``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libdak_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the sm_100a kernels cannot be built")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(out: Path, inputs: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def build(verbose: bool = False, force: bool = False, jobs: int | None = None) -> Path:
    """Compiles every .cu file of csrc/ and links libdak_b200.so; returns its path."""
    nvcc = nvcc_path()
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [REPO_DIR / "include" / "dak_b200.h"]
    if not force and not _stale(LIB_PATH, deps):
        return LIB_PATH
    obj_dir = PKG_DIR / "_build"
    obj_dir.mkdir(exist_ok=True)
    common = [
        nvcc, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
        "-I", str(REPO_DIR / "include"),
    ]
    if verbose:
        common += ["-Xptxas", "-v"]
    procs = []
    objs = []
    for src in srcs:
        obj = obj_dir / (src.stem + ".o")
        objs.append(obj)
        if not force and not _stale(obj, [src] + deps[len(srcs):]):
            continue
        cmd = common + ["-c", str(src), "-o", str(obj)]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if verbose or p.returncode != 0:
            sys.stdout.write(f"== {src.name}\n{out}")
        if p.returncode != 0:
            failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed for {', '.join(failed)}")
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stdout.write(r.stdout)
        raise RuntimeError("linking libdak_b200.so failed")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose", action="store_true", help="show nvcc/ptxas output (-Xptxas -v)")
    ap.add_argument("--force", action="store_true", help="rebuild everything")
    args = ap.parse_args()
    path = build(verbose=args.verbose, force=args.force)
    print(path)


if __name__ == "__main__":
    main()
