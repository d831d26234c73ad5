"""Native fixture reader / writer (bgtq_fixture_*) against the reference's fixture format
(tests/oracles/fixture.py:13-49).  CPU only.

* tests/golden/fixture_format/low_d16 was written by the reference's own write_fixture
  (tests/golden/make_fixture_format.py): the native reader returns its arrays exactly.
* Files the native writer makes are read back exactly, and a restatement of read_fixture
  (below: JSON + SHA-256 + NumPy) accepts them with the same arrays.
* Corrupt files raise LayoutError with read_fixture's messages.
"""
import hashlib
import json

import numpy as np
import pytest

from bgtq import LayoutError
from bgtq.fixture import DTYPES, read_fixture, write_fixture
from conftest import GOLDEN, load_mixed


def restated_read(path):
    """tests/oracles/fixture.py:read_fixture, restated."""
    meta = json.loads(path.read_text(encoding="utf-8"))
    assert meta["version"] in (1, 2) and meta["endianness"] == "little"
    payload = path.with_name(meta["binary"]).read_bytes()
    assert len(payload) == meta["byte_length"] and hashlib.sha256(payload).hexdigest() == meta["sha256"]
    out = {}
    for name, d in meta["arrays"].items():
        dt = DTYPES[d["dtype"]]
        n = int(np.prod(d["shape"])) * dt.itemsize
        assert d["offset"] % 4 == 0 and d["nbytes"] == n and d["offset"] + n <= len(payload)
        out[name] = np.frombuffer(payload, dt, n // dt.itemsize, d["offset"]).reshape(d["shape"])
    return meta, out


def test_reads_reference_written_fixture():
    meta, arrays = read_fixture(GOLDEN / "fixture_format" / "low_d16.json")
    z = load_mixed("low_d16")
    assert meta["name"] == "low_d16" and meta["version"] == 2 and meta["rows"] == 5
    expect = {"original": z["original"].astype(np.float32), "codes": z["codes"].astype(np.uint8),
              "norm_bits": z["norm_bits"].astype(np.uint16), "packed": z["packed"].astype(np.uint8),
              "permutation": z["permutation"].astype(np.uint32),
              "reconstructed_f16": z["reconstructed_f16"].astype(np.float16)}
    assert list(arrays) == list(expect)
    for k, v in expect.items():
        assert arrays[k].dtype == v.dtype
        np.testing.assert_array_equal(arrays[k], v)


def test_write_read_round_trip(tmp_path):
    rng = np.random.default_rng(2)
    arrays = {"a": ("f32", rng.standard_normal((3, 5))), "b": ("u8", rng.integers(0, 256, 7)),
              "c": ("f16", rng.standard_normal((2, 2, 3))), "d": ("u16", rng.integers(0, 65536, 9)),
              "e": ("u32", rng.integers(0, 2**32, 4, dtype=np.uint64)), "empty": ("f32", np.zeros((0, 4)))}
    meta = {"name": "round trip", "version": 2, "nested": {"x": [1, 2.5, "y"], "ok": True, "none": None},
            "text": "quote \" slash \\ newline \n"}
    path = tmp_path / "sub" / "case.json"
    write_fixture(path, meta, arrays)
    got_meta, got = read_fixture(path)
    ref_meta, ref = restated_read(path)
    for k, (dt, v) in arrays.items():
        want = np.asarray(v, dtype=DTYPES[dt])
        np.testing.assert_array_equal(got[k], want)
        np.testing.assert_array_equal(ref[k], want)
        assert got[k].shape == want.shape
    for k, v in meta.items():
        assert got_meta[k] == v == ref_meta[k]
    # payload layout: every array on a 4-byte boundary, total padded to 4
    assert all(d["offset"] % 4 == 0 for d in ref_meta["arrays"].values()) and ref_meta["byte_length"] % 4 == 0


def test_rejections_match_read_fixture(tmp_path):
    path = tmp_path / "f.json"
    write_fixture(path, {"version": 1}, {"a": ("f32", np.arange(4)), "b": ("u8", np.arange(3))})
    good_json, good_bin = path.read_text(), path.with_suffix(".bin").read_bytes()

    bad = bytearray(good_bin)
    bad[0] ^= 1
    path.with_suffix(".bin").write_bytes(bytes(bad))
    with pytest.raises(LayoutError, match="Fixture payload length/hash mismatch"):
        read_fixture(path)
    path.with_suffix(".bin").write_bytes(good_bin)

    m = json.loads(good_json)
    m["version"] = 3
    path.write_text(json.dumps(m))
    with pytest.raises(LayoutError, match="Unsupported fixture format"):
        read_fixture(path)
    m["version"], m["endianness"] = 1, "big"
    path.write_text(json.dumps(m))
    with pytest.raises(LayoutError, match="Unsupported fixture format"):
        read_fixture(path)
    m["endianness"] = "little"
    m["arrays"]["b"]["offset"] = 18       # not 4-byte aligned
    path.write_text(json.dumps(m))
    with pytest.raises(LayoutError, match="Invalid array descriptor: b"):
        read_fixture(path)
    m["arrays"]["b"]["offset"], m["arrays"]["a"]["nbytes"] = 16, 12   # nbytes != prod(shape) * itemsize
    path.write_text(json.dumps(m))
    with pytest.raises(LayoutError, match="Invalid array descriptor: a"):
        read_fixture(path)
    path.write_text(good_json)
    assert list(read_fixture(path)[1]) == ["a", "b"]
