"""Build libunltd_gpu.so in-tree: nvcc, sm_100a only.

    python unltd-inference_b200/build.py [--force] [-j N]

Objects go to unltd-inference_b200/_build/, the library to
unltd-inference_b200/lib/libunltd_gpu.so. Rebuilds a translation unit when
it or any header under csrc/ or include/ is newer than its object.
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
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libunltd_gpu.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I" + os.path.join(REPO, "include"),
    "-DUNLTD_BUILD",
]


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found")
    return p


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(
        os.path.join(REPO, "include", "*.h")
    )


def _needs(obj: str, src: str, hdr_mtime: float) -> bool:
    if not os.path.exists(obj):
        return True
    m = os.path.getmtime(obj)
    return m < os.path.getmtime(src) or m < hdr_mtime


def _compile(src: str, obj: str, extra: list[str]) -> str:
    cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}")
    return r.stderr


def build(force: bool = False, jobs: int = 8, verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr_m = max([os.path.getmtime(h) for h in _headers()] + [0.0])
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.splitext(os.path.basename(s))[0] + ".o")
        objs.append(o)
        if force or _needs(o, s, hdr_m):
            todo.append((s, o))
    extra = ["-Xptxas", "-v"] if ptxas_v else []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = {ex.submit(_compile, s, o, extra): s for s, o in todo}
            for f in cf.as_completed(futs):
                msg = f.result()
                if verbose and msg:
                    print(f"== {os.path.basename(futs[f])}\n{msg}")
    if force or todo or not os.path.exists(LIB):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcuda", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true", help="print ptxas -v resource usage")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v, ptxas_v=a.v))


if __name__ == "__main__":
    sys.exit(main())
