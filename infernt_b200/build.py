"""Builds infernt_b200/lib/libinfernt_b200.so (sm_100a) in the source tree.

Every .cu under csrc/ is compiled by nvcc for sm_100a; every .cpp under
csrc/ and csrc/host/ by nvcc's host compiler.  Objects go to _build/ and
are rebuilt when a source or any header is newer.  The CUDA runtime is
linked statically (nvcc's default), so the library does not depend on the
runtime version other libraries in the process load.

    python -m infernt_b200.build          # or: python infernt_b200/build.py
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libinfernt_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
CU_FLAGS = ARCH + ["-lineinfo", "--expt-relaxed-constexpr"]


def _sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    cpp = sorted(glob.glob(os.path.join(CSRC, "*.cpp")) + glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    return cu, cpp


def _headers():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _obj(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _stale(src, obj, newest_header):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _compile(src, verbose):
    obj = _obj(src)
    flags = COMMON + (CU_FLAGS if src.endswith(".cu") else ARCH + ["-x", "c++"])
    cmd = [NVCC] + flags + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("compile failed: %s\n%s%s" % (src, r.stdout, r.stderr))
    return obj


def build(verbose=False, jobs=None):
    """Compile stale objects and relink the shared library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    cu, cpp = _sources()
    srcs = cu + cpp
    newest_header = max([os.path.getmtime(h) for h in _headers()] + [0])
    todo = [s for s in srcs if _stale(s, _obj(s), newest_header)]
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        list(ex.map(lambda s: _compile(s, verbose), todo))
    objs = [_obj(s) for s in srcs]
    if todo or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC, "-shared"] + ARCH + ["-o", LIB] + objs + ["-Xlinker", "-Bsymbolic", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed\n%s%s" % (r.stdout, r.stderr))
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
