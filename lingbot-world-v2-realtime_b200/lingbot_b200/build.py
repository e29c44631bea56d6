"""Build liblbq.so (the CUDA kernels + C ABI) in-tree with nvcc for sm_100a.

    python -m lingbot_b200.build          # from lingbot-world-v2-realtime_b200/
"""
import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(ROOT, "csrc")
LIB = os.path.join(PKG_DIR, "liblbq.so")
SOURCES = ["quant.cu", "attn.cu", "capi.cu", "noalloc.cu", "peer.cu", "capi_peer.cu"]
HEADERS = ["lbq_ptx.cuh", "lbq_kernels.h", "lbq_peer.cuh", os.path.join("..", "..", "include", "lbq.h")]


def nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def flags(extra=()):
    return ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
            "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
            *extra]


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, extra=()):
    """Compile each .cu to an object, then link the shared library. Returns the library path."""
    if not force and not stale():
        return LIB
    objs = []
    build_dir = os.path.join(ROOT, "_build")
    os.makedirs(build_dir, exist_ok=True)
    for src in SOURCES:
        obj = os.path.join(build_dir, src.replace(".cu", ".o"))
        cmd = [nvcc(), *flags(extra), "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
           *objs, "-o", tmp]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True,
                extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else ()))
