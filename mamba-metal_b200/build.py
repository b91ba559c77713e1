"""Build libmamba_b200.so (sm_100a) in-tree.

    python mamba-metal_b200/build.py [--force] [--verbose-ptxas]

Each csrc/*.cu is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a, no fast-math) into _build/, then
linked into mamba-metal_b200/lib/libmamba_b200.so against the CUDA runtime
and cuBLAS.  The output library travels with the source tree; nothing is
installed elsewhere.
"""
import concurrent.futures
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libmamba_b200.so")
INCLUDE = os.path.join(ROOT, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
                     "-I", INCLUDE, "-I", CSRC, "--expt-relaxed-constexpr"]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _compile(src, force, ptxas_verbose):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(
            os.path.getmtime(src), _newest(headers())):
        return obj, ""
    cmd = [NVCC] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s%s" % (src, r.stdout, r.stderr))
    return obj, r.stderr


def build(force=False, ptxas_verbose=False, jobs=None):
    """Compile every kernel source for sm_100a and link the shared library."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sources()
    logs = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
        results = list(ex.map(lambda s: _compile(s, force, ptxas_verbose), srcs))
    objs = [o for o, _ in results]
    logs = [l for _, l in results if l]
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + [
            "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcublas", "-lcudart", "-ldl",
            "-Xlinker", "-rpath=" + os.path.join(CUDA_HOME, "lib64")]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s%s" % (r.stdout, r.stderr))
    return LIB, "\n".join(logs)


if __name__ == "__main__":
    lib, log = build(force="--force" in sys.argv, ptxas_verbose="--verbose-ptxas" in sys.argv)
    if log:
        print(log)
    print(lib)
