"""Build the in-tree CUDA library ``trnsparse_b200/libtrnsparse_b200.so``.

Every ``csrc/*.cu`` file is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``) and linked into one shared library that
exports the C ABI declared in ``include/trnsparse_b200.h``. Objects are
rebuilt when their source or any header is newer; compilation runs in
parallel. Usage: ``python -m trnsparse_b200.build [--force] [--verbose]``.
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
INCLUDE = ROOT / "include"
OBJ = PKG / "_build"
LIB = PKG / "libtrnsparse_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-rdc=true",
    "-I",
    str(INCLUDE),
    "-I",
    str(CSRC),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the trnsparse_b200 CUDA library cannot be built")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, verbose: bool, extra: list[str]) -> None:
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout, r.stderr, flush=True)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr_t = _headers_mtime()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    todo = []
    objs = []
    for s in srcs:
        o = OBJ / (s.stem + ".o")
        objs.append(o)
        if force or ptxas_verbose or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr_t):
            todo.append((s, o))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            futs = [ex.submit(_compile, s, o, verbose or ptxas_verbose, extra) for s, o in todo]
            for f in futs:
                f.result()
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills/smem per kernel")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
