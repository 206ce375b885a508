"""B200 fused-MoE expert engine.

Importing the package loads the in-tree native libraries:

* ``libmoe_b200.so`` (CUDA kernels + C ABI, include/moe_b200.h), exposed via
  :mod:`moe_ascend_opt_b200.capi`;
* ``_nanovllm_b200.so``, which registers the reference's operator surface
  ``torch.classes.nanovllm.MoEInfer`` and ``torch.ops.nanovllm.moe_forward*``
  (Int8-gemm/nanovllm_ops.cpp:349-431) for CUDA tensors.

There is no CPU implementation: without the built libraries the import fails.
Run ``python moe_ascend_opt_b200/build.py`` (or ``__graft_entry__.build()``).
"""
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmoe_b200.so")
TORCH_LIB_PATH = os.path.join(_HERE, "_nanovllm_b200.so")

for _p in (LIB_PATH, TORCH_LIB_PATH):
    if not os.path.exists(_p):
        raise ImportError(f"{_p} is missing: build the CUDA extension with `python moe_ascend_opt_b200/build.py`")

torch.ops.load_library(TORCH_LIB_PATH)

Q8_0, Q4_0, AWQ = 0, 1, 2

from . import capi  # noqa: E402,F401
