"""The C ABI library on the CPU: it loads, exports every declared symbol, and its
host-only entry points (table validation, allocator) behave like the reference.

Mirrors the reference's layout validation (src/webgpu/layout.ts:8-23), PackedKeys group
checks (src/runtime/packed-keys.ts:15-23, tests/webgpu/optimized-test.ts:72-75) and the
allocator tests (tests/test_allocator.py).
"""
import itertools
import re

import numpy as np
import pytest

import oracle
from bgtq import _lib, layout
from bgtq.layout import BlockGTQParameters, tables, validate_layout
from conftest import GOLDEN, ROOT, allocator_cases, load_config, load_mixed, mixed_cases, params_tables


def declared_symbols():
    text = (ROOT / "include" / "bgtq.h").read_text()
    return sorted(set(re.findall(r"\b(bgtq_[a-z_0-9]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 25
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and header disagree"
    assert b"sm_100a" in lib.bgtq_version()
    assert lib.bgtq_status_string(_lib.ECAPACITY) == b"capacity exceeded"


@pytest.mark.parametrize("name", mixed_cases())
def test_validate_accepts_reference_tables_and_derives_ranges(name):
    z = load_mixed(name)
    p, cfg, tab = params_tables(z)
    info, ranges = validate_layout(cfg, tab)
    assert (info.dim, info.groups, info.nibble_dims, info.row_bytes) == (p.dim, p.groups, p.nibble_dims, p.row_bytes)
    assert info.logical_row_bytes == int(z["logical_row_bytes"])
    # odd number of 32-bit words (conflict-free shared-memory row reads), covering the row
    assert info.device_row_stride % 4 == 0 and (info.device_row_stride // 4) % 2 == 1
    assert info.logical_row_bytes <= info.device_row_stride < info.logical_row_bytes + 8
    np.testing.assert_array_equal(ranges, oracle.group_ranges(p.group_of, p.rotation, p.dim))


def test_tables_flattening_matches_reference_calibration_format():
    z = np.load(GOLDEN / "smollm2_heads.npz")
    for i in range(int(z["heads"])):
        config, table = z[f"h{i}_config"], z[f"h{i}_table"]
        p = BlockGTQParameters.from_tables(config, table)
        c2, t2 = tables(p)
        np.testing.assert_array_equal(c2, config)
        np.testing.assert_array_equal(t2, table)
        info, ranges = validate_layout(config, table)
        np.testing.assert_array_equal(ranges, z[f"h{i}_ranges"])
        assert info.dim == 64 and info.row_bytes == config[2]


def _bad(p, **changes):
    q = BlockGTQParameters(**{**p.__dict__, **changes})
    return tables(q)


def test_validate_rejections():
    z = load_mixed("mixed_d64")
    p, cfg, tab = params_tables(z)
    cases = {
        "Invalid Block-GTQ layout": [dict(dim=130), dict(groups=9), dict(norm_stride=p.groups - 1),
                                     dict(nibble_dims=3), dict(row_bytes=1), dict(max_centroids=1)],
        "Invalid calibration table shape": [dict(permutation=np.zeros(p.dim, np.uint32)),
                                            dict(group_of=np.full(p.dim, 9, np.uint32)),
                                            dict(offsets=p.offsets[:-1])],
        "Code LUT incompatible": [dict(code_lut=np.full_like(p.code_lut, 255))],
        "Nonfinite": [dict(offsets=np.where(np.arange(p.dim) == 3, np.nan, p.offsets).astype(np.float32))],
    }
    for message, changes in cases.items():
        for ch in changes:
            c2, t2 = _bad(p, **ch)
            with pytest.raises(_lib.LayoutError, match=message):
                validate_layout(c2, t2)
    # optimized-test.ts:72-75: a nonzero off-group rotation entry is rejected, not truncated
    rot = p.rotation.reshape(p.dim, p.dim).copy()
    other = int(np.nonzero(p.group_of != p.group_of[0])[0][0])
    rot[other, 0] = 0.01
    with pytest.raises(_lib.LayoutError, match="Off-group transform is nonzero"):
        validate_layout(*_bad(p, rotation=rot.reshape(-1)))
    g = p.group_of.copy()
    g[0], g[-1] = g[-1], g[0]
    with pytest.raises(_lib.LayoutError, match="Non-contiguous"):
        validate_layout(*_bad(p, group_of=g))
    with pytest.raises(_lib.LayoutError):
        validate_layout(cfg[:5], tab)


def test_native_allocator_matches_golden_and_oracle():
    for case in allocator_cases():
        got = layout.allocate_bits(case["scores"], case["budget"], case["min_bits"], case["max_bits"])
        np.testing.assert_array_equal(got, case["expected"])
    for scores in itertools.product((0, 1, 4), repeat=3):
        for budget in range(0, 14):
            np.testing.assert_array_equal(layout.allocate_bits(scores, budget, 1, 4),
                                          oracle.allocate_bits(scores, budget, 1, 4))
    rng = np.random.default_rng(0)
    for _ in range(20):
        s = rng.exponential(size=32).astype(np.float32)
        np.testing.assert_array_equal(layout.allocate_bits(s, 128), oracle.allocate_bits(s, 128))
    z = load_config("config4")
    np.testing.assert_array_equal(layout.allocate_bits(z["scores"], 128, 1, 8), z["widths"])


def test_host_validation_happens_before_device_work():
    """Object creation with invalid arguments fails on the host, without a GPU."""
    with pytest.raises(_lib.RangeError):
        from bgtq import FP16Keys
        FP16Keys(3, 10)
    with pytest.raises(_lib.RangeError):
        from bgtq import Values
        Values(64, 0)
