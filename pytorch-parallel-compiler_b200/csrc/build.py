"""Builds libwidek.so (all CUDA kernels + the C-ABI) for sm_100a with nvcc.

Usage: python build.py [--force] [--jobs N]

Every ``*.cu`` file in this directory is compiled to an object under
``../_build/`` and the objects are linked into
``../wide_compiler/_lib/libwidek.so``. An object is rebuilt when its source or
any header here (or ``include/widek.h``) is newer than it. The CUDA runtime is
linked statically; the driver API is reached through
``cudaGetDriverEntryPoint``, so the library needs no ``-lcuda`` at link time.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
REPO_ROOT = os.path.dirname(PKG_ROOT)
BUILD_DIR = os.path.join(PKG_ROOT, "_build")
LIB_DIR = os.path.join(PKG_ROOT, "wide_compiler", "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libwidek.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", os.path.join(REPO_ROOT, "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH")


def _headers() -> list[str]:
    return glob.glob(os.path.join(HERE, "*.cuh")) + [os.path.join(REPO_ROOT, "include", "widek.h")]


def _stale(src: str, obj: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _compile(src: str, obj: str, extra: list[str]) -> tuple[str, int, str]:
    cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    p = subprocess.run(cmd, capture_output=True, text=True)
    return src, p.returncode, p.stdout + p.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    objs, todo = [], []
    for src in sources:
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(src, obj, newest_header):
            todo.append((src, obj))
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = [ex.submit(_compile, s, o, extra or []) for s, o in todo]
            failed = []
            for f in cf.as_completed(futs):
                src, rc, out = f.result()
                if rc != 0:
                    failed.append((src, out))
                elif verbose and out.strip():
                    print(out)
        if failed:
            msg = "\n".join(f"--- {s}\n{o}" for s, o in failed)
            raise RuntimeError(f"nvcc failed for {len(failed)} file(s):\n{msg}")
    if todo or not os.path.exists(LIB_PATH):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc()] + ARCH_FLAGS + ["-shared", "-o", tmp] + objs
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError("link failed:\n" + p.stdout + p.stderr)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, jobs=a.jobs, verbose=a.verbose or a.ptxas_v, extra=extra))
    return 0


if __name__ == "__main__":
    sys.exit(main())
