"""Build recipe of the oracle's compiled CPU code (test / benchmark infrastructure only):
oracle/cpu_gemv.c -> oracle/_build/libcpu_gemv.so with gcc (POSIX threads). The output is git-ignored
and travels with the tree; nothing in the product links it."""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "cpu_gemv.c"
OUT = HERE / "_build" / "libcpu_gemv.so"
# x86-64-v3 (AVX2 + FMA): vectorised, and runs on any current x86 server host
FLAGS = ["-O3", "-march=x86-64-v3", "-pthread", "-shared", "-fPIC", "-std=c11"]


def build(force: bool = False) -> Path:
    if not force and OUT.exists() and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
    OUT.parent.mkdir(exist_ok=True)
    r = subprocess.run([cc, *FLAGS, str(SRC), "-o", str(OUT)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building {SRC.name} failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(force=True))
