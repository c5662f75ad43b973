"""Builds libsheafb200.so in-tree with nvcc for sm_100a.

    python -m sheaf_b200.build [--force]

Objects go to sheaf_b200/_build/, the library to sheaf_b200/libsheafb200.so.
Rebuilds a translation unit when it or any header is newer than its object.
"""
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsheafb200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_LIB = "/usr/local/cuda/lib64"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cpp")) + glob.glob(os.path.join(CSRC, "kernels", "*.cu")))


def headers():
    return glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))


def _obj(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    return os.path.join(BUILD, rel + ".o")


def _compile(src, force):
    obj = _obj(src)
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj, None
    cmd = [NVCC] + ARCH + COMMON + ["-c", src, "-o", obj]
    if src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"] if os.environ.get("SHEAF_B200_PTXAS_V") else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    if r.stderr.strip() and os.environ.get("SHEAF_B200_PTXAS_V"):
        sys.stderr.write(r.stderr)
    return obj, None


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        results = list(ex.map(lambda s: _compile(s, force), srcs))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + [
        "-L", CUDA_LIB, "-lnvrtc", "-lcudart", "-ldl", "-lpthread",
        "-Xlinker", f"-rpath,{CUDA_LIB}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
