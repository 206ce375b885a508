"""In-tree build of the engine's native libraries.

* ``libmoe_b200.so``     -- CUDA kernels + the C ABI of include/moe_b200.h,
  compiled by nvcc for sm_100a only.
* ``_nanovllm_b200.so``  -- the PyTorch binding (``torch.ops.nanovllm`` /
  ``torch.classes.nanovllm``), linked against libmoe_b200.so.

Both land next to this file so that they travel with the source tree.
Rebuilds only what is older than its sources.  ``python
moe_ascend_opt_b200/build.py`` runs it (a plain script: the package itself needs
the libraries to import).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(ROOT, "_build", "obj")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = os.path.join(HERE, "libmoe_b200.so")
TORCH_LIB = os.path.join(HERE, "_nanovllm_b200.so")


def _newer(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def build_capi(verbose_ptxas: bool = False) -> str:
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(ROOT, "include", "moe_b200.h")]
    os.makedirs(OBJ, exist_ok=True)
    objs = []
    for src in cu:
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if _newer(obj, [src] + headers):
            cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-c", src, "-o", obj]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd)
    if _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", *objs, "-o", LIB, "-lcudart"])
    return LIB


def build_torch_binding() -> str:
    import torch

    src = os.path.join(CSRC, "torch_binding.cpp")
    if not _newer(TORCH_LIB, [src, LIB, os.path.join(ROOT, "include", "moe_b200.h")]):
        return TORCH_LIB
    tdir = os.path.dirname(torch.__file__)
    inc = [os.path.join(tdir, "include"), os.path.join(tdir, "include", "torch", "csrc", "api", "include"),
           os.path.join(CUDA_HOME, "include"), sysconfig.get_paths()["include"]]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{i}" for i in inc], src, "-o", TORCH_LIB,
           f"-L{HERE}", "-lmoe_b200", "-Wl,-rpath,$ORIGIN",
           f"-L{os.path.join(tdir, 'lib')}", f"-Wl,-rpath,{os.path.join(tdir, 'lib')}",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           f"-L{os.path.join(CUDA_HOME, 'lib64')}", "-lcudart"]
    _run(cmd)
    return TORCH_LIB


def build(verbose_ptxas: bool = False) -> None:
    build_capi(verbose_ptxas)
    build_torch_binding()


if __name__ == "__main__":
    build(verbose_ptxas="-v" in sys.argv)
