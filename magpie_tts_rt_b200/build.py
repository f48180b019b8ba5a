"""Build the sm_100a shared library ``libmagpie_tts_rt_b200.so`` in-tree.

nvcc compiles every ``csrc/*.cu`` / ``csrc/*.cpp`` for
``-gencode arch=compute_100a,code=sm_100a`` (nvcc cross-compiles without a
GPU) and links them with the CUDA runtime statically; no other library is
linked (every GEMM is this library's own tcgen05 kernel).  A linker version script
exports only the ``mtt_*`` C symbols declared in ``include/*.h``, as the
reference's plugin library exports only its C ABI
(``cmake/magpie_tts_rt_plugins.map``).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBRARY = os.path.join(HERE, "libmagpie_tts_rt_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "-I" + os.path.join(REPO, "include"), "--expt-relaxed-constexpr"]
# TensorRT (optional): with NvInfer.h found, trt_plugins.cpp's IPluginV3
# creators are compiled in and register_plugins registers them; without it
# (this image) register_plugins reports REGISTRY_UNAVAILABLE.
TENSORRT_DIRS = [d for d in (os.environ.get("TENSORRT_ROOT", ""), "/usr", "/usr/local/tensorrt") if d]


def tensorrt():
    for root in TENSORRT_DIRS:
        for inc in (os.path.join(root, "include"), os.path.join(root, "include", "x86_64-linux-gnu")):
            if os.path.exists(os.path.join(inc, "NvInfer.h")):
                return inc, os.path.join(root, "lib")
    return None


VERSION_SCRIPT = """{
  global:
    mtt_*;
  local:
    *;
};
"""


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, extra):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if _stale(obj, [src] + headers()):
        cmd = [NVCC] + ARCH + COMMON + extra + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    trt = tensorrt()
    if trt is not None:
        extra += ["-DMTT_B200_WITH_TENSORRT", "-I" + trt[0]]
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = list(pool.map(lambda s: _compile(s, extra), srcs))
    if force or _stale(LIBRARY, objs):
        vs = os.path.join(BUILD, "exports.map")
        with open(vs, "w") as fh:
            fh.write(VERSION_SCRIPT)
        cuda_lib = os.path.join(os.path.dirname(os.path.dirname(NVCC)), "lib64")
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIBRARY] + objs + [
            "-L" + cuda_lib, "-Xlinker", "-rpath," + cuda_lib,
            "-Xlinker", "--version-script=" + vs] + (["-L" + trt[1], "-lnvinfer"] if trt is not None else [])
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
