"""Build the in-tree shared library ``libgmdn_b200.so`` for sm_100a.

    python gmdn-gated-muon-deltanet_b200/build.py [--force] [--jobs N]

Every ``csrc/*.cu`` file is compiled by nvcc for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` and linked into
``libgmdn_b200.so`` next to this file.  The library exposes the C ABI of
``include/gmdn_scan.h`` and nothing else; it does not depend on torch.
A file is recompiled only when it or any header it may include is newer than
its object, so repeated calls are cheap.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD = os.path.join(PKG_DIR, "_build")
LIB = os.path.join(PKG_DIR, "libgmdn_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgmdn_b200.so")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(src: str, obj: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _compile(src: str, obj: str, extra: list[str]) -> tuple[str, str]:
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", CSRC, "-I", os.path.join(ROOT, "include"),
           "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
    return src, res.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False,
          extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr_t = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(s, o, hdr_t):
            todo.append((s, o))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for src, log in ex.map(lambda so: _compile(*so, extra or []), todo):
                if verbose and log.strip():
                    print(f"[{os.path.basename(src)}]\n{log}", file=sys.stderr)
    if todo or not os.path.exists(LIB):
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB + ".tmp"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(LIB + ".tmp", LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true",
                    help="print register / shared-memory use of every kernel")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_verbose else []
    print(build(force=args.force or args.ptxas_verbose, jobs=args.jobs,
                verbose=args.verbose or args.ptxas_verbose, extra=extra))


if __name__ == "__main__":
    main()
