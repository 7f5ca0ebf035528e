"""sepia_b200 -- a B200-native (sm_100a) backend for rinaldofesta/sepia's
quantized-matvec / MoE decode hot path.

  csrc/       CUDA kernels + the C ABI (libsepia_cuda.so)
  lib.py      ctypes binding of that ABI (no CPU fallback)
  ops.py      torch-tensor wrappers of the raw-pointer entry points
  synth.py    seeded synthetic weights in the reference's block formats
  moe.py      the HBM-resident expert store and the (expert-sharded) MoE layer
"""
from .lib import LIB_PATH, load  # noqa: F401

__all__ = ["load", "LIB_PATH"]
