"""ctypes binding of libbgtq.so (the C ABI declared in include/bgtq.h).

The library is loaded from this package directory.  There is deliberately no fallback:
if libbgtq.so is missing, importing the binding raises, because every compute path of
this package runs on the GPU through the library.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libbgtq.so"

OK, EINVAL, ECAPACITY, ENONFINITE, EBUSY, ELAYOUT, ETIMEOUT, ECUDA, ENOMEM = range(9)
F16, F32 = 1, 2
KEYS_PACKED, KEYS_FP16, KEYS_COMPRESSED = 1, 2, 3


class BGTQError(Exception):
    """Base class; `status` holds the bgtq_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class RangeError(BGTQError, ValueError):
    """The reference's RangeError: shapes, capacity, positions, non-finite input."""


class LayoutError(RangeError):
    """Invalid Block-GTQ layout or tables (validateLayout / PackedKeys checks)."""


class StateError(BGTQError, RuntimeError):
    """The reference's plain Error: storage not ready, K/V lengths differ."""


class DeviceError(BGTQError, RuntimeError):
    """CUDA failure, allocation failure or a bounded device wait that expired."""


_EXC = {EINVAL: RangeError, ECAPACITY: RangeError, ENONFINITE: RangeError, ELAYOUT: LayoutError,
        EBUSY: StateError, ETIMEOUT: DeviceError, ECUDA: DeviceError, ENOMEM: DeviceError}


class LayoutInfo(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("dim", "groups", "row_bytes", "norm_stride", "nibble_dims", "max_centroids",
                                          "logical_row_bytes", "device_row_stride", "device_scale_stride", "codebooks")]


class Allocation(C.Structure):
    _fields_ = [("name", C.c_char_p), ("role", C.c_char_p), ("bytes", C.c_uint64)]


class DecoderDesc(C.Structure):
    """bgtq_decoder_desc: per-layer arrays are pointers to arrays of device pointers."""
    _fields_ = [(n, C.c_uint32) for n in ("layers", "batch", "hidden", "q_heads", "kv_heads", "head_dim",
                                          "intermediate", "vocab")] + [
        ("rms_eps", C.c_float)] + [(n, C.c_void_p) for n in (
            "inv_freq", "ln1", "qkv_bias", "ln2", "w_qkv", "w_o", "w_gate_up", "w_down", "final_norm", "lm_head",
            "embedding", "attention")] + [("ctas_per_sm", C.c_uint32)]


# (name, restype, argtypes) for every exported symbol declared in include/bgtq.h
P, U32, U64, I32, I64, SZ = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32, C.c_int64, C.c_size_t
SIGNATURES = {
    "bgtq_status_string": (C.c_char_p, [I32]),
    "bgtq_last_error": (C.c_char_p, []),
    "bgtq_version": (C.c_char_p, []),
    "bgtq_allocate_bits": (I32, [P, U32, I64, I32, I32, P]),
    "bgtq_tables_build": (I32, [U32, P, P, U32, U32, U32, P, SZ, P, P, SZ, P]),
    "bgtq_haar_rotation": (I32, [U32, U64, P]),
    "bgtq_optimal_centroids": (I32, [U32, U32, P]),
    "bgtq_set_layout_jit": (I32, [I32]),
    "bgtq_layout_jit_stats": (I32, [P, P]),
    "bgtq_layout_jit_counts": (I32, [P, P, P]),
    "bgtq_layout_jit_prebuild": (I32, [C.c_char_p, U32, P, P, P, P, U32, C.c_int, P, C.c_size_t]),
    "bgtq_layout_jit_prebuilt": (I32, [P]),
    "bgtq_values_read": (I32, [P, U32, U32, U32, P]),
    "bgtq_values_info": (I32, [P, P, P, P, P]),
    "bgtq_keys_layout": (I32, [P, P]),
    "bgtq_model_gemv": (I32, [C.c_int, P, U32, C.c_uint64, U32, P, C.c_float, P, P, U32, P, C.c_uint64, P]),
    "bgtq_decoder_create": (I32, [C.POINTER(DecoderDesc), C.POINTER(P)]),
    "bgtq_decoder_step": (I32, [P, P, P, P, P]),
    "bgtq_decoder_info": (I32, [P, C.POINTER(U32), C.POINTER(U32), C.POINTER(U32)]),
    "bgtq_decoder_trace": (I32, [P, C.c_int, P, U32, C.POINTER(U32)]),
    "bgtq_decoder_destroy": (None, [P]),
    "bgtq_layout_jit_wait": (I32, [U32]),
    "bgtq_fixture_read": (I32, [C.c_char_p, P]),
    "bgtq_fixture_array_count": (I32, [P, P]),
    "bgtq_fixture_array": (I32, [P, U32, P, P, P, P, P, P]),
    "bgtq_fixture_manifest": (I32, [P, P]),
    "bgtq_fixture_destroy": (None, [P]),
    "bgtq_fixture_write": (I32, [C.c_char_p, C.c_char_p, U32, P, P, P, P, P]),
    "bgtq_layout_validate": (I32, [P, SZ, P, SZ, P, C.POINTER(LayoutInfo)]),
    "bgtq_tables_create": (I32, [P, SZ, P, SZ, C.c_int, C.POINTER(P)]),
    "bgtq_tables_info": (I32, [P, C.POINTER(LayoutInfo)]),
    "bgtq_tables_destroy": (None, [P]),
    "bgtq_keys_create": (I32, [C.c_int, P, U32, U32, U32, C.c_int, C.POINTER(P)]),
    "bgtq_keys_destroy": (None, [P]),
    "bgtq_keys_append": (I32, [P, P, C.c_int, C.c_int, U32, U64, U32, U32, U64, P]),
    "bgtq_keys_length": (I32, [P, U32, C.POINTER(U32)]),
    "bgtq_keys_info": (I32, [P, C.POINTER(C.c_int), C.POINTER(U32), C.POINTER(U32), C.POINTER(U32)]),
    "bgtq_keys_read": (I32, [P, U32, U32, U32, P, P]),
    "bgtq_keys_reconstruct": (I32, [P, U32, P, P]),
    "bgtq_keys_allocations": (I32, [P, C.POINTER(Allocation), U32, C.POINTER(U32)]),
    "bgtq_values_create": (I32, [C.c_int, U32, U32, U32, C.c_int, C.POINTER(P)]),
    "bgtq_values_destroy": (None, [P]),
    "bgtq_values_append": (I32, [P, P, C.c_int, C.c_int, U32, U64, U32, U32, U64, P]),
    "bgtq_values_length": (I32, [P, U32, C.POINTER(U32)]),
    "bgtq_attention_create": (I32, [U32, P, P, U32, C.POINTER(P)]),
    "bgtq_attention_destroy": (None, [P]),
    "bgtq_attend": (I32, [P, P, P, C.c_int, U32, U32, U32, P, P, P, C.c_int, P]),
    "bgtq_attention_last_splits": (I32, [P, C.POINTER(U32)]),
    "bgtq_attention_set_splits": (I32, [P, U32]),
    "bgtq_attention_set_schedule": (I32, [P, I32]),
    "bgtq_attention_last_stream_k": (I32, [P, C.POINTER(U32)]),
    "bgtq_attention_last_launches": (I32, [P, C.POINTER(U32)]),
    "bgtq_device_status": (I32, [C.c_int, C.POINTER(U32)]),
    "bgtq_attend_static": (I32, [U32, P, P, P, P, C.c_int, U32, U32, U32, P, P]),
    "bgtq_attend_prefill": (I32, [P, P, U32, U32, U32, U32, U32, P, C.c_int, P]),
    "bgtq_keys_reset": (I32, [P, P]),
    "bgtq_append_kv_rope": (I32, [U32, P, P, P, C.c_uint64, C.c_uint64, U32, U32, U32, U32, U32, P, P]),
    "bgtq_append_kv": (I32, [U32, P, P, P, I32, P, I32, I32, U32, C.c_uint64, U32, U32, C.c_uint64, P]),
    "bgtq_attention_set_prefill_kernel": (I32, [P, U32]),
    "bgtq_attention_set_rope": (I32, [P, P, U32]),
    "bgtq_attention_plan_for_capacity": (I32, [P, C.c_int]),
    "bgtq_keys_sync_lengths": (I32, [P]),
    "bgtq_values_sync_lengths": (I32, [P]),
    "bgtq_values_reset": (I32, [P, P]),
}

_lib = None


def lib() -> C.CDLL:
    """Load (once) and return the library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with "
                              f"`python block-gqt-webgpu_b200/build.py` (no CPU fallback exists)")
        handle = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status != OK:
        message = lib().bgtq_last_error().decode() or lib().bgtq_status_string(status).decode()
        raise _EXC.get(status, BGTQError)(status, message)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
