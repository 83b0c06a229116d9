"""Build the B200 W4A8 library in-tree.

Outputs (next to the Python package, so they travel with the source tree):
  w4a8_fp8_wmma/libw4a8_b200.so  — the C-ABI library (every CUDA kernel, sm_100a)
  w4a8_fp8_wmma/_C.so            — the torch op shim over the C ABI

Usage: python rdna4-vllm_b200/build.py [--force]
Compilation is incremental on file modification times and runs in parallel.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
PKG = os.path.join(HERE, "w4a8_fp8_wmma")
OBJ = os.path.join(HERE, "_build")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["act_quant.cu", "moe_align.cu", "gemm_mma.cu", "gemv_stream.cu", "gemm_tc.cu", "reduce.cu", "moe_layer.cu", "moe_decode.cu", "ep_dispatch.cu",
              "router.cu", "capi.cu"]
LIB = os.path.join(PKG, "libw4a8_b200.so")
SHIM = os.path.join(PKG, "_C.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
    "-diag-suppress", "186",
]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs + [os.path.join(INCLUDE, "w4a8_b200.h")]


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def _compile_cu(src: str, force: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src).replace(".cu", ".o"))
    if force or _newer(obj, [src] + _headers()):
        _run([NVCC, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj])
    return obj


def build_lib(force: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in CU_SOURCES if os.path.exists(os.path.join(CSRC, s))]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile_cu(s, force), srcs))
    if force or _newer(LIB, objs):
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", LIB,
              "-lcudart"])
    return LIB


def build_shim(force: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "torch_binding.cpp")
    if not (force or _newer(SHIM, [src, LIB, os.path.join(INCLUDE, "w4a8_b200.h")])):
        return SHIM
    incs = cpp_extension.include_paths() + [os.path.join(CUDA_HOME, "include"), INCLUDE,
                                            sysconfig.get_paths()["include"]]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-fPIC", "-shared", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H=0", "-w"]
    for i in incs:
        cmd += ["-I", i]
    cmd += [src, "-o", SHIM, "-L", torch_lib, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_cuda", "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart",
            "-L", PKG, "-lw4a8_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    _run(cmd)
    return SHIM


def build(force: bool = False) -> None:
    build_lib(force)
    build_shim(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(LIB)
    print(SHIM)
