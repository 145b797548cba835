"""Build libqf2b200.so in-tree from quantfun2_b200/csrc/*.cu for sm_100a.

Each translation unit is compiled with nvcc (-gencode arch=compute_100a,code=sm_100a)
into quantfun2_b200/_build/, then linked into quantfun2_b200/libqf2b200.so with the
CUDA runtime linked statically, so the library carries no torch dependency.
Objects are rebuilt when their source or any header is newer.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libqf2b200.so"
INCLUDE = PKG.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-I" + str(INCLUDE),
]


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool, extra: list[str], force: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj
    cmd = [NVCC, *CFLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile and link.  Extra nvcc flags (e.g. -D tuning macros) may be passed in the
    QF2_NVCC_FLAGS environment variable; they force a full rebuild."""
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    flags = os.environ.get("QF2_NVCC_FLAGS", "").split()
    extra = (["-Xptxas", "-v"] if ptxas_info else []) + flags
    stamp = BUILD / "flags.txt"
    changed = not stamp.exists() or stamp.read_text() != " ".join(flags)
    force = changed or ptxas_info
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose or ptxas_info, extra, force), srcs))
    stamp.write_text(" ".join(flags))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest or force:
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
