"""Builds libgptoss.so (the C ABI of include/gptoss.h) for sm_100a, in-tree.

    python gptoss-infer_b200/build.py [--force]

Each csrc/*.cu compiles to _build/*.o with nvcc (-gencode arch=compute_100a,code=sm_100a, -lineinfo, no fast-math:
E8M0 scale 0 decodes to the fp32 subnormal 2^-127, which flush-to-zero would destroy), then links into
gptoss-infer_b200/lib/libgptoss.so. Objects are rebuilt only when a source or header is newer.
"""
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
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libgptoss.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-Wall", "--expt-relaxed-constexpr",
         "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src, obj, verbose):
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if verbose else ""


def build(force=False, verbose=False):
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0)
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if force or verbose or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, newest_header):
            jobs.append((s, o))
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for log in ex.map(lambda j: _compile(*j, verbose), jobs):
            if log:
                print(log, file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or jobs or not LIB.exists():
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcuda", "-lcublas",
               "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/shared-memory usage")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
