"""Builds libl0b200.so (the C-ABI backend) in-tree with nvcc for sm_100a.

Usage: python -m l0llm_b200.build [--force] [--jobs N]

Objects go to l0llm_b200/_build/ and the library to l0llm_b200/libl0b200.so. Sources are rebuilt
when they, or any header under csrc/ or include/, are newer than their object.
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
LIB = PKG / "libl0b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden,-O3",
    f"-I{ROOT / 'include'}",
    f"-I{CSRC}",
]


def _sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def _headers_mtime() -> float:
    hs = [*CSRC.glob("*.h"), *CSRC.glob("*.cuh"), *(ROOT / "include").glob("*.h")]
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, hdr_mtime: float) -> Path:
    obj = BUILD / (src.name + ".o")
    if not force and obj.exists():
        om = obj.stat().st_mtime
        if om >= src.stat().st_mtime and om >= hdr_mtime:
            return obj
    cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [NVCC, "-x", "cu", *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    hdr = _headers_mtime()
    jobs = jobs or min(8, os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hdr), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcuda", "-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print(f"built {LIB}")
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args()
    build(force=a.force, jobs=a.jobs, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
