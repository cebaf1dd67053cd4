"""Build the sm_100a C-ABI library ``lib/libsdl_b200.so`` from ``csrc/*.cu``.

Run ``python build_lib.py`` (or call :func:`build`).  Each translation unit is
compiled by nvcc for ``arch=compute_100a,code=sm_100a`` with ``-lineinfo`` and
linked into one shared object; CUDA's runtime is linked statically so the
library only needs the NVIDIA driver at run time.  Objects are rebuilt only
when a source or header is newer than the object.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from typing import List

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
OBJDIR = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIBNAME = "libsdl_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
BASE_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O2",
    "-I" + INCLUDE,
    "-I" + CSRC,
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH")


def lib_path() -> str:
    return os.path.join(LIBDIR, LIBNAME)


def _headers() -> List[str]:
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdrs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hdrs


def _stale(target: str, deps: List[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(nvcc: str, src: str, obj: str, verbose_ptxas: bool) -> str:
    cmd = [nvcc, *ARCH_FLAGS, *BASE_FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed for {}:\n{}\n{}".format(src, res.stdout, res.stderr))
    return res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> str:
    """Compile every ``csrc/*.cu`` and link ``lib/libsdl_b200.so``; return its path."""
    nvcc = nvcc_path()
    os.makedirs(OBJDIR, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    sources = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    headers = _headers()
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(OBJDIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    logs = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, nvcc, s, o, verbose_ptxas): s for s, o in jobs}
            for fut in cf.as_completed(futs):
                logs.append((futs[fut], fut.result()))
    out = lib_path()
    if force or jobs or _stale(out, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", out, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError("link failed:\n{}\n{}".format(res.stdout, res.stderr))
    if not quiet or verbose_ptxas:
        for src, log in logs:
            if log.strip():
                print("== {}\n{}".format(os.path.basename(src), log))
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true", help="rebuild every object")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers / spills / smem per kernel")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose_ptxas=args.ptxas_v, quiet=False)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
