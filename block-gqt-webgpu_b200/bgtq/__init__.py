"""Block-GTQ key-cache compression on B200: K encode + compressed-K GQA attention.

Host-side mirror of the reference's TypeScript surface (amw720386/block-gqt-webgpu:
src/webgpu/layout.ts, src/runtime/*.ts, src/attention/*.ts) over the C ABI of
libbgtq.so (include/bgtq.h).  All compute runs in hand-written sm_100a kernels; there is
no CPU fallback - a missing library raises ImportError on first use.
"""
from ._lib import (BGTQError, DeviceError, LayoutError, RangeError, StateError, LIB_PATH, lib)
from .layout import (BlockGTQParameters, allocate_bits, build_tables, haar_rotation, optimal_centroids, tables,
                     validate_layout)
from .runtime import CompressedKeys, FP16Keys, PackedKeys, Values, append_kv
from .attention import AttentionEngine, AttentionSession, GroupedAttention, OptimizedAttention

__all__ = ["BGTQError", "DeviceError", "LayoutError", "RangeError", "StateError", "LIB_PATH", "lib",
           "BlockGTQParameters", "allocate_bits", "build_tables", "haar_rotation", "optimal_centroids", "tables", "validate_layout", "CompressedKeys", "FP16Keys", "append_kv",
           "PackedKeys", "Values", "AttentionEngine", "AttentionSession", "GroupedAttention", "OptimizedAttention",
           "device_status"]


def device_status(device: int = 0) -> int:
    """Device status word (0 = no kernel reported a timeout or bad length)."""
    import ctypes as C
    from . import _lib
    v = C.c_uint32()
    _lib.call("bgtq_device_status", device, C.byref(v))
    return v.value
