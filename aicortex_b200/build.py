"""Builds the CUDA extension libaicortex_b200.so in-tree for sm_100a.

Every .cu file under csrc/ is compiled with nvcc (-gencode
arch=compute_100a,code=sm_100a, --use_fast_math as the reference build uses)
and linked with a static CUDA runtime into aicortex_b200/libaicortex_b200.so,
which is what the Python package and the tests load. Objects go to
aicortex_b200/_build/ and are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libaicortex_b200.so"

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = [
    "-std=c++17", "-O3", "--use_fast_math", "-lineinfo", *ARCH,
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", str(ROOT / "include"), "-I", str(CSRC),
]


def _newest_header() -> float:
    hdrs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hdrs), default=0.0)


def _compile(src: Path, hdr_time: float, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_time):
        return obj
    cmd = [NVCC, *CFLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr_time = _newest_header()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, hdr_time, verbose), srcs))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
