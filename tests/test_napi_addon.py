"""The Node-API addon (block-gqt-webgpu_b200/napi/bgtq_napi.c) - the drop-in the reference's
TypeScript classes call - compiled and exercised without Node.js.

Neither this image nor the GPU box has Node, so the addon is compiled here with the
declarations of tests/napi/node_api.h (Node-API's documented signatures) and linked with
a stand-in runtime (tests/napi/fake_napi.c) that implements those functions over a small
value model.  The tests call the addon's exports the way JavaScript would, with typed
arrays and numbers, and compare with the C ABI / Python package: layouts, the allocator
and the table builder on the CPU; stores, appends, reads and attention on the GPU.  Errors
must surface as the reference's classes: RangeError for shapes, capacity and layouts.
"""
import ctypes as C
import subprocess

import numpy as np
import pytest

import bgtq
from bgtq import _lib
from conftest import GOLDEN, ROOT, load_config, params_tables

ADDON = ROOT / "block-gqt-webgpu_b200" / "napi" / "bgtq_napi.c"
TYPES = {np.dtype(np.uint8): 1, np.dtype(np.uint16): 4, np.dtype(np.int32): 5, np.dtype(np.uint32): 6,
         np.dtype(np.float32): 7}
NP_OF = {v: k for k, v in TYPES.items()}


class JsError(Exception):
    pass


class JsRangeError(JsError):
    pass


class JsValue:
    """A value the addon returned (a napi_value of the stand-in runtime)."""

    def __init__(self, ptr):
        self.ptr = ptr


class Addon:
    """The addon's exports behind the stand-in runtime."""

    def __init__(self, so):
        self.h = C.CDLL(str(so))
        P = C.c_void_p
        for name, res, args in [("fake_env", P, []), ("fake_module", P, [P]), ("fake_null", P, []),
                                ("fake_bool", P, [C.c_int]), ("fake_number", P, [C.c_double]),
                                ("fake_typed", P, [C.c_int, P, C.c_size_t]), ("fake_array", P, [P, C.c_size_t]),
                                ("fake_call", P, [P, P, C.c_char_p, P, C.c_size_t]),
                                ("fake_exception", C.c_int, [P, C.c_char_p, C.c_size_t]),
                                ("fake_kind", C.c_int, [P]), ("fake_get_number", C.c_double, [P]),
                                ("fake_get", P, [P, C.c_char_p]),
                                ("fake_typed_info", C.c_int, [P, C.POINTER(P), C.POINTER(C.c_size_t)]),
                                ("fake_gc", C.c_int, [P])]:
            f = getattr(self.h, name)
            f.restype, f.argtypes = res, args
        self.env = self.h.fake_env()
        self.exports = JsValue(self.h.fake_module(self.env))
        self.keep = []

    def arg(self, x):
        """A JS value for x; typed arrays view the NumPy buffer (no copy), so results written
        into an output array show up in the caller's array."""
        if isinstance(x, JsValue):
            return x.ptr
        if x is None:
            return self.h.fake_null()
        if isinstance(x, bool):
            return self.h.fake_bool(int(x))
        if isinstance(x, (int, float)):
            return self.h.fake_number(float(x))
        if isinstance(x, np.ndarray):
            a = np.ascontiguousarray(x)
            self.keep.append(a)
            return self.h.fake_typed(TYPES[a.dtype], a.ctypes.data, a.size)
        if isinstance(x, list):
            vals = (C.c_void_p * len(x))(*[self.arg(e) for e in x])
            self.keep.append(vals)
            return self.h.fake_array(vals, len(x))
        raise TypeError(f"no JavaScript value for {type(x)}")

    def __call__(self, name, *args):
        argv = (C.c_void_p * max(1, len(args)))(*[self.arg(a) for a in args])
        r = self.h.fake_call(self.env, self.exports.ptr, name.encode(), argv, len(args))
        msg = C.create_string_buffer(1024)
        kind = self.h.fake_exception(self.env, msg, 1024)
        if kind:
            raise (JsRangeError if kind == 2 else JsError)(msg.value.decode())
        return JsValue(r)

    def typed(self, v):
        data, n = C.c_void_p(), C.c_size_t()
        t = self.h.fake_typed_info(v.ptr, C.byref(data), C.byref(n))
        assert t >= 0, "not a typed array"
        dt = NP_OF[t]
        return np.ctypeslib.as_array(C.cast(data, C.POINTER(np.ctypeslib.as_ctypes_type(dt))), (n.value,)).copy() \
            if n.value else np.zeros(0, dt)

    def get(self, obj, name):
        return JsValue(self.h.fake_get(obj.ptr, name.encode()))

    def number(self, v):
        return self.h.fake_get_number(v.ptr)


@pytest.fixture(scope="module")
def addon(tmp_path_factory):
    out = tmp_path_factory.mktemp("napi") / "bgtq_napi_test.so"
    libdir = _lib.LIB_PATH.parent
    cmd = ["gcc", "-std=c11", "-O1", "-Wall", "-Wextra", "-Werror", "-Wno-unused-parameter", "-shared", "-fPIC",
           "-I", str(ROOT / "tests" / "napi"), "-I", str(ROOT / "include"), str(ADDON),
           str(ROOT / "tests" / "napi" / "fake_napi.c"), "-o", str(out), f"-L{libdir}", "-lbgtq",
           f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return Addon(out)


def test_addon_exports_every_function(addon):
    for name in ("validateLayout", "allocateBits", "buildTables", "packedKeysCreate", "fp16KeysCreate",
                 "valuesCreate", "keysAppend", "valuesAppend", "keysLength", "valuesLength", "keysRead",
                 "attentionCreate", "attend", "attendPrefill", "destroy", "deviceStatus"):
        assert addon.h.fake_kind(addon.get(addon.exports, name).ptr) == 8, name   # a function


@pytest.mark.parametrize("name", ["config1", "config4"])
def test_validate_layout_matches_the_library(addon, name):
    p, cfg, tab = params_tables(load_config(name))
    r = addon("validateLayout", cfg, tab)
    info, ranges = bgtq.validate_layout(cfg, tab)
    for js, field in [("dim", "dim"), ("groups", "groups"), ("rowBytes", "row_bytes"), ("normStride", "norm_stride"),
                      ("nibbleDims", "nibble_dims"), ("maxCentroids", "max_centroids")]:
        assert addon.number(addon.get(r, js)) == getattr(info, field), js
    np.testing.assert_array_equal(addon.typed(addon.get(r, "ranges")), ranges)


def test_validate_layout_throws_the_references_range_errors(addon):
    p, cfg, tab = params_tables(load_config("config4"))
    bad = cfg.copy()
    bad[0] = 63                                           # odd head dim
    with pytest.raises(JsRangeError):
        addon("validateLayout", bad, tab)
    with pytest.raises(JsRangeError):
        addon("validateLayout", cfg, tab[:-3])            # short table
    with pytest.raises(JsRangeError, match="validateLayout"):
        addon("validateLayout", tab, cfg)                 # wrong typed-array kinds


def test_allocator_and_table_builder_through_the_addon(addon):
    z = np.load(GOLDEN / "qwen_calibration.npz")
    for i in (0, int(np.argmax(z["norm_stride"]))):
        scores = z["scores"][i].astype(np.float32)
        widths = addon.typed(addon("allocateBits", scores, 128, 1, 8))
        np.testing.assert_array_equal(widths, bgtq.allocate_bits(scores, 128, 1, 8))
        np.testing.assert_array_equal(widths, z["widths"][i])
        t = addon("buildTables", widths.astype(np.int32), 2, 0, int(z["norm_stride"][i]))
        cfg, tab = bgtq.build_tables(widths, rotation_threshold=2, norm_stride=int(z["norm_stride"][i]))
        np.testing.assert_array_equal(addon.typed(addon.get(t, "config")), cfg)
        np.testing.assert_array_equal(addon.typed(addon.get(t, "table")), tab)


@pytest.mark.gpu
def test_stores_and_attention_through_the_addon(addon, cuda):
    """PackedKeys / Values / OptimizedAttention driven through the addon equal the library's
    own Python surface on the same inputs (one sequence, as the reference's session)."""
    import oracle
    from bgtq import synthetic
    p, cfg, tab = params_tables(load_config("config4"))
    rng = np.random.default_rng(41)
    T, R, d = 700, 3, 64
    k16 = synthetic.profiled(rng, T, d).astype(np.float16).view(np.uint16)
    v32 = rng.standard_normal((T, d)).astype(np.float32)
    keys = addon("packedKeysCreate", cfg, tab, 1024)
    vals = addon("valuesCreate", True, d, 1024)
    addon("keysAppend", keys, k16[:500].reshape(-1))
    addon("keysAppend", keys, k16[500:].reshape(-1))
    addon("valuesAppend", vals, v32.reshape(-1))
    assert addon.number(addon("keysLength", keys, 0)) == T == addon.number(addon("valuesLength", vals, 0))
    rd = addon("keysRead", keys, 0)
    ref = oracle.encode(cfg, tab, k16)
    np.testing.assert_array_equal(addon.typed(addon.get(rd, "packed")).reshape(T, -1), ref["packed"])
    np.testing.assert_array_equal(addon.typed(addon.get(rd, "scales")).reshape(T, -1), ref["scales"])
    att = addon("attentionCreate", [keys], [vals], R)
    q = synthetic.profiled(rng, R, d)
    pos = np.array([0, 350, T - 1], np.uint32)
    out = np.zeros((R, d), np.float32)
    logits = np.zeros((R, T), np.float32)
    probs = np.zeros((R, T), np.float32)
    addon("attend", att, q.reshape(-1), pos, True, R, out.reshape(-1), logits.reshape(-1), probs.reshape(-1))
    kh = oracle.reconstruct(cfg, tab, ref["packed"], ref["scales"])
    lg, pr, o = oracle.attention(q, kh, v32, pos, True)
    np.testing.assert_allclose(out, o, atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(probs, pr, atol=1e-6, rtol=1e-4)
    # errors as the reference throws them: positions past the keys, K/V length mismatch
    with pytest.raises(JsRangeError):
        addon("attend", att, q.reshape(-1), np.array([0, 1, T], np.uint32), True, R, np.zeros(R * d, np.float32))
    with pytest.raises(JsRangeError, match="whole nonempty rows"):
        addon("keysAppend", keys, k16[:1, :5].reshape(-1))
    addon("keysAppend", keys, k16[:1].reshape(-1))
    with pytest.raises(JsError):
        addon("attend", att, q.reshape(-1), None, False, R, np.zeros(R * d, np.float32))
    addon("destroy", att)
    with pytest.raises(JsRangeError):
        addon("attend", att, q.reshape(-1), None, False, R, np.zeros(R * d, np.float32))   # destroyed handle
    assert addon.h.fake_gc(addon.env) >= 3                  # finalizers free what destroy() did not
    assert addon.number(addon("deviceStatus", 0)) == 0


@pytest.mark.gpu
def test_prefill_through_the_addon(addon, cuda):
    """attendPrefill: the model path's causal prefill chunk through the addon equals the
    Python surface's result bit for bit (same kernel, same inputs)."""
    from bgtq import GroupedAttention, PackedKeys, Values, synthetic
    p, cfg, tab = params_tables(load_config("config4"))
    rng = np.random.default_rng(42)
    T, G, d = 300, 3, 64
    k16 = synthetic.profiled(rng, T, d).astype(np.float16).view(np.uint16)
    v16 = rng.standard_normal((T, d)).astype(np.float16).view(np.uint16)
    keys = addon("packedKeysCreate", cfg, tab, 512)
    vals = addon("valuesCreate", False, d, 512)
    addon("keysAppend", keys, k16.reshape(-1))
    addon("valuesAppend", vals, v16.reshape(-1))
    att = addon("attentionCreate", [keys], [vals], G)
    q = synthetic.profiled(rng, T * G, d).reshape(1, T, G, d)
    got = np.zeros((1, T, G, d), np.float32)
    addon("attendPrefill", att, q.reshape(-1), 0, T, G, got.reshape(-1))
    pk, pv = PackedKeys((cfg, tab), 512), Values(d, 512, "f16")
    pk.append(k16)
    pv.append(v16)
    np.testing.assert_array_equal(got, GroupedAttention([pk], [pv], G).prefill(q))
