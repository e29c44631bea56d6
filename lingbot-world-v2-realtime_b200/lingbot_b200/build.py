"""Build liblbq.so (the CUDA kernels + C ABI) in-tree with nvcc for sm_100a.

    python -m lingbot_b200.build [--debug]   # from lingbot-world-v2-realtime_b200/
"""
import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(ROOT, "csrc")
LIB = os.path.join(PKG_DIR, "liblbq.so")
DEBUG_LIB = os.path.join(PKG_DIR, "liblbq_debug.so")
SOURCES = ["quant.cu", "attn.cu", "fp8lin.cu", "capi.cu", "noalloc.cu", "peer.cu", "capi_peer.cu"]
HEADERS = ["lbq_ptx.cuh", "lbq_kernels.h", "lbq_peer.cuh", os.path.join("..", "..", "include", "lbq.h")]


def nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def flags(extra=()):
    return ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
            "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
            *extra]


def stale(lib=None):
    lib = LIB if lib is None else lib
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, extra=(), debug=False):
    """Compile each .cu to an object, then link the shared library. Returns the library path.
    debug=True builds liblbq_debug.so instead: the same kernels with the device-side index checks
    (-DLBQ_DEBUG=1) that record a 0x3xx status code where the index arithmetic goes wrong; the
    package loads it when LBQ_DEBUG_LIB=1."""
    lib = DEBUG_LIB if debug else LIB
    if not force and not stale(lib):
        return lib
    objs = []
    build_dir = os.path.join(ROOT, "_build", "debug" if debug else "release")
    os.makedirs(build_dir, exist_ok=True)
    if debug:
        extra = ("-DLBQ_DEBUG=1", *extra)
    for src in SOURCES:
        obj = os.path.join(build_dir, src.replace(".cu", ".o"))
        cmd = [nvcc(), *flags(extra), "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = lib + ".tmp"
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
           *objs, "-o", tmp]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, debug="--debug" in sys.argv,
                extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else ()))
