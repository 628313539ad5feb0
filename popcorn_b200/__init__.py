"""popcorn_b200 — B200 (sm_100a) decode-step kernels behind Popcorn's API.

The kernels and the C ABI live in ``_lib/libpopcorn_cuda.so`` (sources in
``csrc/``, ABI in ``include/popcorn_cuda.h``); ``api`` mirrors the
reference's Swift surface in Python over that ABI; ``decode`` composes the
decode layer and stack used by the benchmark (dense, and 4-bit affine);
``safetensors`` reads weight archives; ``tp`` runs tensor-parallel decode.
"""
from .api import (Access, AffineQuantizedTensor, AttentionMask, DataType, FixedScratch, Kernel,
                  KernelCommandEncoder, KernelLibrary, KernelScratchAllocator, Kernels, PeerGroup, PopcornError,
                  ScratchPool, ScratchSpec, Tensor, device_error_check)

__all__ = ["Access", "AffineQuantizedTensor", "AttentionMask", "DataType", "FixedScratch", "Kernel",
           "KernelCommandEncoder", "KernelLibrary", "KernelScratchAllocator", "Kernels", "PeerGroup", "PopcornError",
           "ScratchPool", "ScratchSpec", "Tensor", "device_error_check"]
