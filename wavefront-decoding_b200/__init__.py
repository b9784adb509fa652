"""wavefront_decoding_b200 — B200-native (sm_100a) wavefront attention and KV-slot
kernels for wavefront decoding of looped LMs, behind a C ABI (include/wfd_b200.h).

Modules:
  attention   reference-compatible attention surface (attn_varlen, attn_dense,
              attn_cutoff_multi, ...) and the slot-native `wave_attn`
  kv_cache    SlotKVCache: per-(slot, sequence) KV storage with device lengths
  runtime     workspace / error word / stream plumbing
  build       nvcc recipe for libwfd_b200.so
"""
from . import _abi  # noqa: F401
from ._abi import WfdError, load as load_library  # noqa: F401

__all__ = ["WfdError", "load_library"]
