"""Build the sampler's C-ABI shared library (libmxs.so) in-tree with nvcc.

Only sm_100a code is generated. The library links the CUDA runtime statically
and exports exactly the functions of include/mxs_sampler.h.
    python minxfmr.cpp_b200/mxs_build.py [--verbose]
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(OUT_DIR, "libmxs.so")
# phase-timer build (-DMXS_PROFILE) for kernel analysis; never loaded by the product path
PROF_LIB = os.path.join(OUT_DIR, "libmxs_prof.so")
SOURCES = ["mxs_sampler.cu", "mxs_stream.cu", "mxs_api.cu", "mxs_noalloc.cu", "mxs_multi.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # every double operation of the draw must round exactly as the reference's
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-shared", "-cudart", "static", "-ldl",
]


def build(verbose=False, force=False, profile=False):
    lib = PROF_LIB if profile else LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [
        os.path.join(HERE, "..", "include", "mxs_sampler.h")]
    if (not force and os.path.exists(lib)
            and os.path.getmtime(lib) >= max(os.path.getmtime(d) for d in deps)):
        return lib
    cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if verbose else []) + (["-DMXS_PROFILE"] if profile else []) + \
        [os.path.join(CSRC, s) for s in SOURCES] + ["-o", lib]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode:
        raise RuntimeError(f"nvcc failed building {lib}")
    return lib


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True, profile="--profile" in sys.argv))
