"""Fixture files of the reference's tests, read and written natively (bgtq_fixture_*).

Same surface as tests/oracles/fixture.py:13-49 of the reference: ``write_fixture(path,
metadata, arrays)`` with ``arrays = {name: (dtype, data)}`` and ``read_fixture(path) ->
(metadata, arrays)``; dtypes f32 / u32 / u8 / f16 / u16; read errors raise LayoutError with
read_fixture's messages.
"""
from __future__ import annotations

import ctypes as C
import json

import numpy as np

from . import _lib

DTYPES = {"f32": np.dtype("<f4"), "u32": np.dtype("<u4"), "u8": np.dtype("u1"),
          "f16": np.dtype("<f2"), "u16": np.dtype("<u2")}


def write_fixture(path, metadata, arrays) -> None:
    names, dts, ndims, shapes, datas, keep = [], [], [], [], [], []
    for name, (dtype, data) in arrays.items():
        a = np.ascontiguousarray(np.asarray(data, dtype=DTYPES[dtype]))
        shp = (C.c_uint64 * max(1, a.ndim))(*a.shape)
        keep += [a, shp]
        names.append(name.encode())
        dts.append(dtype.encode())
        ndims.append(a.ndim)
        shapes.append(C.cast(shp, C.c_void_p))
        datas.append(a.ctypes.data)
    n = len(names)
    _lib.call("bgtq_fixture_write", str(path).encode(), json.dumps(metadata, allow_nan=False).encode(), n,
              (C.c_char_p * max(1, n))(*names), (C.c_char_p * max(1, n))(*dts), (C.c_uint32 * max(1, n))(*ndims),
              (C.c_void_p * max(1, n))(*shapes), (C.c_void_p * max(1, n))(*datas))


def read_fixture(path):
    h = C.c_void_p()
    _lib.call("bgtq_fixture_read", str(path).encode(), C.byref(h))
    try:
        text = C.c_char_p()
        _lib.call("bgtq_fixture_manifest", h, C.byref(text))
        meta = json.loads(text.value.decode("utf-8"))
        count = C.c_uint32()
        _lib.call("bgtq_fixture_array_count", h, C.byref(count))
        arrays = {}
        for i in range(count.value):
            name, dtype = C.c_char_p(), C.c_char_p()
            ndim, shape, data, nbytes = C.c_uint32(), C.POINTER(C.c_uint64)(), C.c_void_p(), C.c_uint64()
            _lib.call("bgtq_fixture_array", h, i, C.byref(name), C.byref(dtype), C.byref(ndim), C.byref(shape),
                      C.byref(data), C.byref(nbytes))
            dt = DTYPES[dtype.value.decode()]
            shp = tuple(shape[k] for k in range(ndim.value))
            buf = (C.c_char * nbytes.value).from_address(data.value) if nbytes.value else b""
            arrays[name.value.decode()] = np.frombuffer(bytes(buf), dt).reshape(shp).copy()
        return meta, arrays
    finally:
        _lib.lib().bgtq_fixture_destroy(h)
