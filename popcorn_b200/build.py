"""Build recipe of the CUDA library ``popcorn_b200/_lib/libpopcorn_cuda.so``.

Every ``csrc/*.cu`` file is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into one shared
library with the CUDA runtime linked statically. The library exports the C
ABI declared in ``include/popcorn_cuda.h`` and nothing else; it has no
dependency on torch or Python.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_lib")
OBJ = os.path.join(OUT, "obj")
LIB = os.path.join(OUT, "libpopcorn_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I" + os.path.join(ROOT, "include"),
]


def _headers():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp"))
    hs.append(os.path.join(ROOT, "include", "popcorn_cuda.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src, extra):
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _headers()):
        return obj
    cmd = [NVCC, *FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, " ".join(cmd), r.stderr))
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas=False, jobs=None):
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
               "-Xcompiler", "-fPIC", "-o", LIB, *objs, "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (" ".join(cmd), r.stderr))
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
