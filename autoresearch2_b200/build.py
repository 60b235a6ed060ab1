"""Build libsparseffn.so (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

Each csrc/*.cu file is compiled to an object in parallel, then linked into
autoresearch2_b200/libsparseffn.so with the CUDA runtime linked statically,
so the library loads on machines without a GPU driver (symbol checks) and
needs no JIT cache at run time.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
OUT = os.path.join(PKG, "libsparseffn.so")
BUILD_DIR = os.path.join(PKG, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math: it flushes denormals to zero, and the pack/mask/gradient
# kernels must reproduce IEEE results bit for bit.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-Xptxas", "-O3",
              "--expt-relaxed-constexpr"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _compile(src, verbose):
    obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
    deps = [src] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    deps.append(os.path.join(os.path.dirname(PKG), "include", "sparseffn.h"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose=False, force=False):
    """Compile every csrc/*.cu for sm_100a and link libsparseffn.so."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    if force:
        for f in os.listdir(BUILD_DIR):
            os.remove(os.path.join(BUILD_DIR, f))
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if os.path.exists(OUT) and not force and \
            os.path.getmtime(OUT) >= max(os.path.getmtime(o) for o in objs):
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
