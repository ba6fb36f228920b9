"""Build the sampler's C-ABI shared library (libmxs.so) in-tree with nvcc.

Only sm_100a code is generated. Each translation unit compiles to its own
object (in parallel, rebuilt only when it or a header is newer); the library
links the CUDA runtime statically and exports exactly the functions of
include/mxs_sampler.h.
    python minxfmr.cpp_b200/mxs_build.py [--verbose] [--profile]
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(OUT_DIR, "libmxs.so")
# phase-timer build (-DMXS_PROFILE) for kernel analysis; never loaded by the product path
PROF_LIB = os.path.join(OUT_DIR, "libmxs_prof.so")
SOURCES = ["mxs_sampler.cu", "mxs_stream.cu", "mxs_api.cu", "mxs_noalloc.cu", "mxs_multi.cu", "mxs_hidden.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
COMPILE_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # every double operation of the draw must round exactly as the reference's
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
]
LINK_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static", "-ldl"]


def _run(cmd, verbose):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
    return r.returncode


def build(verbose=False, force=False, profile=False):
    lib = PROF_LIB if profile else LIB
    obj_dir = os.path.join(OUT_DIR, "obj_prof" if profile else "obj")
    os.makedirs(obj_dir, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if not f.endswith(".cu")] + [
        os.path.join(HERE, "..", "include", "mxs_sampler.h")]
    newest_header = max(os.path.getmtime(h) for h in headers)
    extra = (["-Xptxas", "-v"] if verbose else []) + (["-DMXS_PROFILE"] if profile else [])

    def obj_of(s):
        return os.path.join(obj_dir, s.replace(".cu", ".o"))

    def stale(s):
        o = obj_of(s)
        src = os.path.join(CSRC, s)
        return force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(src), newest_header)

    todo = [s for s in SOURCES if stale(s)]
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        rcs = list(ex.map(lambda s: _run([NVCC] + COMPILE_FLAGS + extra + ["-c", os.path.join(CSRC, s), "-o",
                                                                         obj_of(s)], verbose), todo))
    if any(rcs):
        raise RuntimeError(f"nvcc failed building {lib}")
    objs = [obj_of(s) for s in SOURCES]
    if todo or not os.path.exists(lib) or os.path.getmtime(lib) < max(os.path.getmtime(o) for o in objs):
        if _run([NVCC] + LINK_FLAGS + objs + ["-o", lib], verbose):
            raise RuntimeError(f"nvcc failed linking {lib}")
    return lib


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv, profile="--profile" in sys.argv))
