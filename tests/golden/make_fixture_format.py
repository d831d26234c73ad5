"""Write tests/golden/fixture_format/low_d16.{json,bin} with the reference's own fixture writer.

Run in a container that has the reference checkout (it is not needed afterwards):

    python tests/golden/make_fixture_format.py --reference <path to block-gqt-webgpu>

The arrays are those of tests/golden/mixed/low_d16.npz (the reference's fixtures/mixed/low_d16
re-saved), written by tests/oracles/fixture.py:write_fixture, so the native reader
(bgtq_fixture_read) is pinned against a file the reference produced.
"""
import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    from tests.oracles.fixture import write_fixture
    z = np.load(HERE / "mixed" / "low_d16.npz")
    arrays = {"original": ("f32", z["original"]), "codes": ("u8", z["codes"]), "norm_bits": ("u16", z["norm_bits"]),
              "packed": ("u8", z["packed"]), "permutation": ("u32", z["permutation"]),
              "reconstructed_f16": ("f16", z["reconstructed_f16"])}
    write_fixture(HERE / "fixture_format" / "low_d16.json", {"name": "low_d16", "version": 2, "rows": 5, "dim": 16},
                  arrays)


if __name__ == "__main__":
    main()
