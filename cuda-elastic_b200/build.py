"""Builds libce_b200.so (the C ABI of include/ce_b200.h) for sm_100a.

Each csrc/*.cu file is compiled to an object under _build/ with nvcc
(-gencode arch=compute_100a,code=sm_100a -lineinfo), then linked into
cuda-elastic_b200/libce_b200.so with the CUDA runtime linked statically.
Objects are rebuilt only when a source or header is newer. Nothing here
needs a GPU: nvcc cross-compiles.
"""
import concurrent.futures
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libce_b200.so")
HOST = os.path.join(PKG, "host")
# Drop-in front ends (host C++ over the C ABI): executable -> sources in host/.
EXECUTABLES = {"llama2c_b200": ["llama2c_b200.cpp", "llama2c_check.cpp"],
               "decoder_b200": ["decoder_b200.cpp", "decoder_check.cpp", "lp_front.cpp"]}

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
          "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]
# Files whose arithmetic order is part of their contract: no contraction of
# a multiply and an add into an FMA.
NO_FMAD = {"simt_gemm.cu", "decoder.cu"}


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    out = [os.path.join(ROOT, "include", "ce_b200.h")]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return out


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose=False, extra=()):
    name = os.path.basename(src)
    obj = os.path.join(BUILD, name + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    cmd = [nvcc(), "-c", src, "-o", obj] + ARCH + COMMON + list(extra)
    if name in NO_FMAD:
        cmd += ["--fmad=false"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {name}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr)
    return obj


def build(verbose=False, ptxas_verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, extra), sources))
    if _stale(LIB, objs):
        cmd = [nvcc(), "-shared", "-o", LIB] + objs + ARCH + ["-cudart", "static", "-lpthread", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    for exe, srcs in EXECUTABLES.items():
        out = os.path.join(PKG, exe)
        paths = [os.path.join(HOST, f) for f in srcs]
        deps = paths + [LIB] + [os.path.join(HOST, f) for f in os.listdir(HOST) if f.endswith(".h")]
        if _stale(out, deps):
            cmd = [nvcc(), "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"), "-I", HOST,
                   "-o", out] + paths + ["-L", PKG, "-lce_b200", "-Xlinker", "-rpath,$ORIGIN",
                                         "-cudart", "static", "-lpthread"]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"build of {exe} failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_verbose="-v" in sys.argv))
