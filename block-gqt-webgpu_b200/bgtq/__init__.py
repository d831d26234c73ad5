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
           "device_status", "set_layout_jit", "layout_jit_stats",
           "layout_jit_counts", "layout_jit_wait"]


def set_layout_jit(on) -> None:
    """Layout-specialised decode attention kernels (bgtq_set_layout_jit): True = every launch,
    False = never, "auto" (the default) = launches of more than one wave of CTAs."""
    from . import _lib
    _lib.call("bgtq_set_layout_jit", 2 if on == "auto" else 1 if on else 0)


def layout_jit_stats() -> tuple[int, int]:
    """(specialised kernels built, layouts that failed to build) in this process."""
    import ctypes as C
    from . import _lib
    b, f = C.c_uint32(), C.c_uint32()
    _lib.call("bgtq_layout_jit_stats", C.byref(b), C.byref(f))
    return b.value, f.value


def layout_jit_counts() -> dict:
    """{"compiled": cubins ready, "loaded": kernels loaded by a launch, "failed": keys that
    failed to build} for the layout-specialised attention kernels of this process."""
    import ctypes as C
    from . import _lib
    c, l, f = C.c_uint32(), C.c_uint32(), C.c_uint32()
    _lib.call("bgtq_layout_jit_counts", C.byref(c), C.byref(l), C.byref(f))
    return {"compiled": c.value, "loaded": l.value, "failed": f.value}


def layout_jit_wait(timeout_s: float = 300.0) -> bool:
    """Wait for the queued background compiles of layout-specialised attention kernels and
    load what they built (call outside a graph capture); False if the time ran out."""
    from . import _lib
    status = _lib.lib().bgtq_layout_jit_wait(max(0, min(int(timeout_s * 1000), 2**32 - 1)))
    if status == _lib.ETIMEOUT:
        return False
    _lib.check(status)
    return True


def device_status(device: int = 0) -> int:
    """Device status word (0 = no kernel reported a timeout or bad length)."""
    import ctypes as C
    from . import _lib
    v = C.c_uint32()
    _lib.call("bgtq_device_status", device, C.byref(v))
    return v.value
