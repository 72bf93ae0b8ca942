"""Build libkan_cuda.so (sm_100a) in-tree: metal-kans_b200/metal_kans/_lib/libkan_cuda.so.

    python metal-kans_b200/build.py [--force] [-j N]

Each translation unit is compiled by nvcc for sm_100a only (no PTX for other targets, no
multi-arch), objects go to metal-kans_b200/_build/, and the shared library links the CUDA
runtime statically (the driver library is resolved at run time through
cudaGetDriverEntryPoint, so the .so needs no libcuda at link time).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT_DIR = os.path.join(HERE, "metal_kans", "_lib")
OUT = os.path.join(OUT_DIR, "libkan_cuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", INCLUDE]
# Host quantisers must round once per source operation (no fma contraction).
CXX_FLAGS = ["-Xcompiler", "-ffp-contract=off"]

# (source, object name, extra defines): the tensor-core kernels are instantiated once per
# (activation dtype, basis), the CUDA-core small-batch kernels once per (activation dtype, batch
# size), in separate translation units so that they compile in parallel.
SOURCES = [("kan_abi.cpp", "kan_abi", []), ("kan_misc.cu", "kan_misc", []),
           ("kan_simt.cu", "kan_simt", []), ("kan_tc.cu", "kan_tc", []),
           ("kan_noalloc.cu", "kan_noalloc", []), ("kan_gemv.cu", "kan_gemv", []),
           ("kan_gemv_cc.cu", "kan_gemv_cc", []), ("kan_backward.cu", "kan_backward", []),
           ("kan_extra.cu", "kan_extra", []), ("kan_train.cu", "kan_train", [])] + [
    ("kan_tc_inst.cu", f"kan_tc_inst_{m}_{b}", [f"-DKAN_TC_MODE={m}", f"-DKAN_TC_BASIS={b}"])
    for m in (1, 2) for b in range(7)] + [
    ("kan_gemv_cc_inst.cu", f"kan_gemv_cc_inst_{m}_{n}", [f"-DKAN_CC_MODE={m}", f"-DKAN_CC_NB={n}"])
    for m in (1, 2) for n in range(1, 5)]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _includes(path, seen=None):
    """The quoted includes of `path`, followed recursively (csrc/ and include/ files only)."""
    import re

    seen = set() if seen is None else seen
    try:
        text = open(path).read()
    except OSError:
        return seen
    for name in re.findall(r'^\s*#\s*include\s+"([^"]+)"', text, re.M):
        dep = os.path.normpath(os.path.join(os.path.dirname(path), name))
        if not os.path.exists(dep):
            dep = os.path.join(INCLUDE, os.path.basename(name))
        if os.path.exists(dep) and dep not in seen:
            seen.add(dep)
            _includes(dep, seen)
    return seen


def _newer(src_paths, target):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(p) > t for p in src_paths)


def _compile(spec, verbose: bool) -> str:
    src, name, defines = spec
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, name + ".o")
    deps = [path] + sorted(_includes(path))
    if not _newer(deps, obj):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_COMMON, *defines, "-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd += CXX_FLAGS
    else:
        cmd += ["-Xptxas", "-v"] if verbose else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    if force:
        for f in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, f))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    if _newer(objs, OUT):
        cmd = [nvcc(), *ARCH, "-shared", "-o", OUT, *objs, "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))
