"""Build libdspark_b200.so in-tree with nvcc for sm_100a.

    python -m mlx_dspark_b200.build            # incremental
    python -m mlx_dspark_b200.build --force    # rebuild everything

Objects go to mlx_dspark_b200/_build/, the shared library to mlx_dspark_b200/libdspark_b200.so.
The CUDA runtime is linked statically and the driver API is reached through
cudaGetDriverEntryPoint, so the library loads on a machine without a GPU driver (the C ABI
symbols can be inspected there) and needs only libcuda.so.1 at the first CUDA call.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libdspark_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-DNDEBUG", f"-I{INCLUDE}",
]
CXX_FLAGS = ["-O2", "-fPIC", "-std=c++17", "-fvisibility=hidden", f"-I{INCLUDE}"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def _sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, verbose: bool, extra: list[str]) -> Path:
    obj = BUILD / (src.name + ".o")
    if (not force and obj.exists()
            and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime())):
        return obj
    nvcc = _nvcc()
    if src.suffix == ".cu":
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [nvcc, "-x", "cu", *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout, r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force or ptxas_info, verbose or ptxas_info, extra), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args(argv)
    lib = build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
