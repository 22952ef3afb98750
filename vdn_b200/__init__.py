"""vdn_b200: B200-native (sm_100a) kernels for the VDN-H3 hybrid DiT block hot path.

Submodules mirror the reference (ec-jt/vdn) op and module API:
  mxfp8_quant, mxfp8_kernels, mxfp8_linear  -- MXFP8 quantiser, producers, GEMM
  paper_factor, linear_attention            -- the VDA branch and its stage ops
  ulysses                                   -- Ulysses sequence parallelism
  block                                     -- the hybrid DiT block used by bench.py
All compute runs in libvdn_b200.so (include/vdn_b200.h); there is no fallback.
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
