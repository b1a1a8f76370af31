"""Build libsgsa_b200.so (sm_100a) in-tree with nvcc.

``python -m sgsa_b200.build`` compiles every ``csrc/*.cu`` to an object in
``sgsa_b200/_build/`` (in parallel, only when the source or a header changed)
and links ``sgsa_b200/_lib/libsgsa_b200.so``.  ``--check`` builds the
bounds-checked debug variant (``-DSGSA_CHECK``, objects in ``_build/check/``)
as ``sgsa_b200/_lib/libsgsa_b200_check.so``.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIBDIR, "libsgsa_b200.so")
LIB_CHECK = os.path.join(LIBDIR, "libsgsa_b200_check.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, verbose: bool, check: bool = False) -> str:
    obj = os.path.join(OBJ, "check" if check else "", os.path.basename(src) + ".o")
    if (os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(src)
            and os.path.getmtime(obj) >= _headers_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *(["-DSGSA_CHECK"] if check else []), "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
    if verbose or "spill" in r.stderr.lower():
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, force: bool = False, check: bool = False) -> str:
    objdir = os.path.join(OBJ, "check") if check else OBJ
    lib = LIB_CHECK if check else LIB
    os.makedirs(objdir, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    if force:
        for o in glob.glob(os.path.join(objdir, "*.o")):
            os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, check), srcs))
    if not os.path.exists(lib) or any(os.path.getmtime(o) > os.path.getmtime(lib) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", lib, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return lib


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv, check="--check" in sys.argv))
