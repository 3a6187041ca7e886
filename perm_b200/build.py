"""Build libcoldpress_cuda.so in-tree for sm_100a.

    python -m perm_b200.build [--force] [-j N]

Each .cu under perm_b200/csrc is compiled separately with nvcc; the units that must
reproduce numpy's float32 results bit for bit (k-quant fit/decode and the error-feedback
sweep) are compiled with -fmad=false so no multiply-add is contracted.  The CUDA runtime is
linked statically, so the library runs inside any process that has a CUDA driver (its kernels
share the device's primary context with PyTorch).
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libcoldpress_cuda.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "-I", os.path.join(ROOT, "include"), "-I", CSRC]
EXACT_UNITS = {"kquant_encode.cu", "kquant_decode.cu", "ef_sweep.cu"}


def nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libcoldpress_cuda.so")


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(ROOT, "include", "coldpress_cuda.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src, force, verbose):
    obj = os.path.join(OBJ, src[:-3] + ".o")
    s = os.path.join(CSRC, src)
    if (not force and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(s), _headers_mtime())):
        return obj, False
    flags = list(COMMON)
    if src in EXACT_UNITS:
        flags += ["-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false"]
    if src == "capi.cu":
        flags += ["-Xcompiler", "-fvisibility=default"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    cmd = [nvcc()] + ARCH + flags + ["-c", s, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj, True


def build(force=False, jobs=8, verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    objs = [o for o, _ in results]
    relink = force or not os.path.exists(LIB) or any(changed for _, changed in results) or \
        max(os.path.getmtime(o) for o in objs) > os.path.getmtime(LIB)
    if relink:
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-ldl", "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))
