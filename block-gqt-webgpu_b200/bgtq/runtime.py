"""Key and value stores over the C ABI, mirroring the reference's runtime classes.

    PackedKeys      src/runtime/packed-keys.ts:7-52    (nibble/byte codes + FP16 scales)
    CompressedKeys  src/runtime/compressed-keys.ts:5-59 (same storage; attention
                    materialises FP32 K first, the reference's "phase 3" path)
    FP16Keys        src/runtime/keys.ts:16-27
    Values          src/runtime/values.ts:3-16 (FP32, as the reference) or FP16 (model V cache)

Differences from the reference surface, all additive: a store may hold several
independent ``sequences`` (one (layer, KV head) of a whole batch); appends accept NumPy
host arrays (validated like the reference: whole non-empty rows, finite values, capacity)
or CUDA tensors already on the store's device (stream-ordered, trusted like the
reference's GPU-resident model path).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .layout import BlockGTQParameters, tables


def _stream_ptr(stream):
    if stream is not None:
        return C.c_void_p(int(stream))
    return None


def _torch_stream(t):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def as_source(values, dim: int):
    """Normalise an append source.

    Returns (ptr, dtype, host, seq_count, count, row_stride, seq_stride, keepalive, stream).
    Accepted: NumPy uint16 (FP16 bits), float16 or float32 arrays; CUDA torch tensors of
    float16 / float32 / int16-as-bits.  Shapes: [n*dim] flat, [count, dim] or
    [seq_count, count, dim] (last dimension contiguous).
    """
    if isinstance(values, np.ndarray) or not hasattr(values, "data_ptr"):
        a = np.asarray(values)
        if a.dtype == np.float16:
            a = a.view(np.uint16)
        if a.dtype == np.uint16:
            dt = _lib.F16
        elif a.dtype == np.float32:
            dt = _lib.F32
        elif a.dtype == np.float64:
            a = a.astype(np.float32)
            dt = _lib.F32
        else:
            raise _lib.RangeError(_lib.EINVAL, f"unsupported append dtype {a.dtype}")
        if a.ndim == 1:
            if a.size == 0 or a.size % dim:
                raise _lib.RangeError(_lib.EINVAL, "append must contain whole nonempty rows")
            a = a.reshape(1, -1, dim)
        elif a.ndim == 2:
            a = a[None]
        if a.ndim != 3 or a.shape[-1] != dim or a.shape[1] == 0:
            raise _lib.RangeError(_lib.EINVAL, "append must contain whole nonempty rows")
        a = np.ascontiguousarray(a)
        return (a.ctypes.data, dt, 1, a.shape[0], a.shape[1], dim, a.shape[1] * dim, a, None)
    t = values
    import torch
    if not t.is_cuda:
        return as_source(t.detach().cpu().numpy(), dim)
    if t.dtype == torch.float16 or t.dtype == torch.int16:
        dt = _lib.F16
    elif t.dtype == torch.float32:
        dt = _lib.F32
    else:
        raise _lib.RangeError(_lib.EINVAL, f"unsupported append dtype {t.dtype}")
    if t.dim() == 2:
        t = t.unsqueeze(0)
    if t.dim() != 3 or t.shape[-1] != dim or t.stride(-1) != 1:
        raise _lib.RangeError(_lib.EINVAL, "append must contain whole rows with a contiguous last dimension")
    return (t.data_ptr(), dt, 0, t.shape[0], t.shape[1], t.stride(1), t.stride(0), t, _torch_stream(t))


class _Store:
    _handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class _Keys(_Store):
    _kind = _lib.KEYS_PACKED
    kind = "block-gtq"

    def __init__(self, parameters, capacity: int, sequences: int = 1, device: int = 0):
        if isinstance(parameters, BlockGTQParameters):
            config, table = tables(parameters)
        else:
            config, table = (np.ascontiguousarray(parameters[0], np.uint32), np.ascontiguousarray(parameters[1], np.float32))
        self.config, self.table = config, table
        t = C.c_void_p()
        _lib.call("bgtq_tables_create", config.ctypes.data, config.size, table.ctypes.data, table.size, device,
                  C.byref(t))
        try:
            info = _lib.LayoutInfo()
            _lib.call("bgtq_tables_info", t, C.byref(info))
            h = C.c_void_p()
            _lib.call("bgtq_keys_create", self._kind, t, info.dim, int(capacity), int(sequences), device, C.byref(h))
        finally:
            _lib.lib().bgtq_tables_destroy(t)
        self._handle = h
        self.info = info
        self.dim, self.capacity, self.sequences, self.device = info.dim, int(capacity), int(sequences), device
        self.row_bytes, self.norm_stride = info.row_bytes, info.norm_stride

    @classmethod
    def create(cls, parameters, capacity: int, sequences: int = 1, device: int = 0):
        return cls(parameters, capacity, sequences, device)

    def append(self, values, seq_first: int = 0, stream=None) -> None:
        ptr, dt, host, seqs, count, rs, ss, keep, ts = as_source(values, self.dim)
        _lib.call("bgtq_keys_append", self._handle, C.c_void_p(ptr), dt, host, count, rs, seq_first, seqs, ss,
                  _stream_ptr(stream if stream is not None else ts))

    def lengths(self, seq: int = 0) -> int:
        n = C.c_uint32()
        _lib.call("bgtq_keys_length", self._handle, seq, C.byref(n))
        return n.value

    def reset(self, stream=None) -> None:
        """Start every sequence over (lengths 0), keeping the capacity (bgtq_keys_reset)."""
        _lib.call("bgtq_keys_reset", self._handle, _stream_ptr(stream))

    @property
    def length(self) -> int:
        return self.lengths(0)

    def ready(self) -> None:
        """packed-keys.ts:50: non-empty storage is required before attention."""
        if not self.length:
            raise _lib.StateError(_lib.EBUSY, "K storage not ready")

    def read(self, seq: int = 0, row0: int = 0, count: int | None = None):
        """(packed rows [count, row_bytes] u8, FP16 scale bits [count, norm_stride] u16)."""
        count = self.lengths(seq) - row0 if count is None else count
        packed = np.zeros((count, self.row_bytes), np.uint8)
        norms = np.zeros((count, self.norm_stride), np.uint16)
        _lib.call("bgtq_keys_read", self._handle, seq, row0, count, packed.ctypes.data, norms.ctypes.data)
        return packed, norms

    def reconstruct(self, seq: int = 0):
        """Materialised FP32 K [length, dim] as a CUDA tensor (CompressedKeys.prepare)."""
        import torch
        n = self.lengths(seq)
        out = torch.empty((n, self.dim), dtype=torch.float32, device=f"cuda:{self.device}")
        _lib.call("bgtq_keys_reconstruct", self._handle, seq, C.c_void_p(out.data_ptr()),
                  C.c_void_p(torch.cuda.current_stream(out.device).cuda_stream))
        return out

    @property
    def allocations(self):
        n = C.c_uint32()
        _lib.call("bgtq_keys_allocations", self._handle, None, 0, C.byref(n))
        arr = (_lib.Allocation * max(n.value, 1))()
        _lib.call("bgtq_keys_allocations", self._handle, arr, n.value, C.byref(n))
        return [dict(name=a.name.decode(), role=a.role.decode(), bytes=int(a.bytes)) for a in arr[:n.value]]

    def destroy(self) -> None:
        if self._handle:
            _lib.lib().bgtq_keys_destroy(self._handle)
            self._handle = None


class PackedKeys(_Keys):
    """PackedKeys (packed-keys.ts): codes + FP16 scales, consumed without reconstruction."""
    _kind = _lib.KEYS_PACKED


class CompressedKeys(_Keys):
    """CompressedKeys (compressed-keys.ts): same storage, attention over materialised FP32 K."""
    _kind = _lib.KEYS_COMPRESSED


class FP16Keys(_Store):
    """FP16Keys (keys.ts:16-27)."""
    kind = "fp16"

    def __init__(self, dim: int, capacity: int, sequences: int = 1, device: int = 0):
        h = C.c_void_p()
        _lib.call("bgtq_keys_create", _lib.KEYS_FP16, None, int(dim), int(capacity), int(sequences), device, C.byref(h))
        self._handle = h
        self.dim, self.capacity, self.sequences, self.device = int(dim), int(capacity), int(sequences), device

    append = _Keys.append
    lengths = _Keys.lengths
    length = _Keys.length
    allocations = _Keys.allocations
    destroy = _Keys.destroy

    def ready(self) -> None:
        if not self.length:
            raise _lib.StateError(_lib.EBUSY, "K storage not ready")

    def read(self, seq: int = 0, row0: int = 0, count: int | None = None):
        count = self.lengths(seq) - row0 if count is None else count
        rows = np.zeros((count, self.dim), np.uint16)
        _lib.call("bgtq_keys_read", self._handle, seq, row0, count, rows.ctypes.data, None)
        return rows


class Values(_Store):
    """Values (values.ts:3-16).  dtype "f32" mirrors the reference; "f16" the model cache."""

    def __init__(self, dim: int, capacity: int, dtype: str = "f32", sequences: int = 1, device: int = 0):
        code = {"f32": _lib.F32, "f16": _lib.F16}.get(dtype)
        if code is None:
            raise _lib.RangeError(_lib.EINVAL, "Invalid V dtype")
        h = C.c_void_p()
        _lib.call("bgtq_values_create", code, int(dim), int(capacity), int(sequences), device, C.byref(h))
        self._handle = h
        self.dim, self.capacity, self.sequences, self.device, self.dtype = int(dim), int(capacity), int(sequences), device, dtype

    def read(self, seq: int = 0, row0: int = 0, count: int | None = None):
        """Rows [row0, row0 + count) of sequence seq as the store holds them: float16 for FP16
        stores, float32 for FP32 stores, [count, dim] (bgtq_values_read)."""
        count = self.lengths(seq) - row0 if count is None else count
        out = np.zeros((count, self.dim), np.float16 if self.dtype == "f16" else np.float32)
        _lib.call("bgtq_values_read", self._handle, seq, row0, count, out.ctypes.data)
        return out

    def append(self, values, seq_first: int = 0, stream=None) -> None:
        ptr, dt, host, seqs, count, rs, ss, keep, ts = as_source(values, self.dim)
        _lib.call("bgtq_values_append", self._handle, C.c_void_p(ptr), dt, host, count, rs, seq_first, seqs, ss,
                  _stream_ptr(stream if stream is not None else ts))

    def lengths(self, seq: int = 0) -> int:
        n = C.c_uint32()
        _lib.call("bgtq_values_length", self._handle, seq, C.byref(n))
        return n.value

    def reset(self, stream=None) -> None:
        """Start every sequence over (lengths 0), keeping the capacity (bgtq_values_reset)."""
        _lib.call("bgtq_values_reset", self._handle, _stream_ptr(stream))

    @property
    def length(self) -> int:
        return self.lengths(0)

    def destroy(self) -> None:
        if self._handle:
            _lib.lib().bgtq_values_destroy(self._handle)
            self._handle = None


def append_kv(keys, values, k, v, seq_first: int = 0, stream=None) -> None:
    """One layer's K/V append for every KV head in one launch (bgtq_append_kv): the per-head
    PackedKeys.append + Values.append of the reference (src/runtime/packed-keys.ts:39-48,
    src/runtime/values.ts:9-14), batched.  k, v: [seq_count, n, heads, dim] or
    [seq_count, heads, dim] (one new token), either CUDA tensors (float16 / float32, the last
    two dimensions contiguous) or host NumPy arrays (uint16 FP16 bits, float16 or float32,
    C-contiguous; uploaded in stream order, so page-locked buffers must not change until the
    stream has passed the call).  keys[h] packed stores, values[h] FP16 stores of one dim."""
    host = isinstance(k, np.ndarray)
    if host != isinstance(v, np.ndarray):
        raise ValueError("k and v must both be host arrays or both CUDA tensors")
    if host:
        def norm(a):
            a = np.ascontiguousarray(a)
            if a.dtype == np.float16:
                a = a.view(np.uint16)
            if a.dtype not in (np.uint16, np.float32):
                raise ValueError("host k / v must be FP16 bits (uint16), float16 or float32")
            return a if a.ndim == 4 else a[:, None]
        k, v = norm(k), norm(v)
        if k.shape != v.shape or k.ndim != 4:
            raise ValueError("k and v must share one shape [seq_count, n, heads, dim]")
        S, n, heads, dim = k.shape
        ptr_k, ptr_v = k.ctypes.data, v.ctypes.data
        dk, dv = (1 if k.dtype == np.uint16 else 2), (1 if v.dtype == np.uint16 else 2)
        rs, ss = heads * dim, n * heads * dim
        st = stream
    else:
        import torch
        if k.dim() == 3:
            k, v = k.unsqueeze(1), v.unsqueeze(1)
        if k.shape != v.shape or k.dim() != 4 or not k.is_cuda or not v.is_cuda:
            raise ValueError("k and v must be CUDA tensors of one shape [seq_count, n, heads, dim]")
        S, n, heads, dim = k.shape
        if k.stride(3) != 1 or k.stride(2) != dim or v.stride(3) != 1 or v.stride(2) != dim or k.stride() != v.stride():
            raise ValueError("k / v layout: [seq_count, n, heads, dim] with contiguous heads x dim")
        dt = {torch.float16: 1, torch.float32: 2}
        if k.dtype not in dt or v.dtype not in dt:
            raise ValueError("k / v must be float16 or float32")
        ptr_k, ptr_v, dk, dv = k.data_ptr(), v.data_ptr(), dt[k.dtype], dt[v.dtype]
        rs, ss = k.stride(1), k.stride(0)
        st = stream if stream is not None else _torch_stream(k)
    if heads != len(keys) or heads != len(values):
        raise ValueError("one key and one value store per head")
    kp = (C.c_void_p * heads)(*[x._handle for x in keys])
    vp = (C.c_void_p * heads)(*[x._handle for x in values])
    _lib.call("bgtq_append_kv", heads, kp, vp, C.c_void_p(ptr_k), dk, C.c_void_p(ptr_v), dv, 1 if host else 0, n, rs,
              seq_first, S, ss, _stream_ptr(st))
