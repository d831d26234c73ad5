"""Build libbgtq.so in-tree for sm_100a with nvcc (no torch extension machinery).

    python block-gqt-webgpu_b200/build.py [--jobs N] [--force] [--no-prebuild]

After the library, the layout-specialised decode-attention kernels of the benchmarked tables
are compiled ahead of time into block-gqt-webgpu_b200/bgtq/aot/ (prebuild()).

Objects go to block-gqt-webgpu_b200/_build/, the library to
block-gqt-webgpu_b200/bgtq/libbgtq.so.  The CUDA runtime is linked statically so the
library does not depend on which libcudart a host process (e.g. PyTorch) loaded.
The encoder and reconstruction translation units are compiled with -fmad=false: their
only fused multiply-adds are explicit fmaf calls, matching the CPU oracle bit for bit.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
OUT_DIR = HERE / "_build"
LIB = HERE / "bgtq" / "libbgtq.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr", "-I", str(SRC)]
STRICT_FP = {"encode.cu", "rows.cu", "step.cu"}


def sources():
    return sorted(list(SRC.glob("*.cu")) + list(SRC.glob("*.cpp")))


def digest(path: Path) -> str:
    h = hashlib.sha256(path.read_bytes())
    for dep in sorted(SRC.glob("*.h")) + sorted(SRC.glob("*.cuh")) + [HERE.parent / "include" / "bgtq.h"]:
        h.update(dep.read_bytes())
    h.update(" ".join(ARCH + COMMON).encode())
    return h.hexdigest()[:16]


def compile_one(src: Path, force: bool, verbose: bool) -> Path:
    obj = OUT_DIR / f"{src.stem}.{digest(src)}.o"
    if obj.exists() and not force:
        return obj
    flags = list(COMMON)
    if src.suffix == ".cu":
        flags += ARCH
        if src.name in STRICT_FP:
            flags += ["-fmad=false"]
        if verbose:
            flags += ["-Xptxas", "-v"]
    cmd = [NVCC, *flags, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        (OUT_DIR / f"{src.stem}.ptxas.txt").write_text(r.stderr)
    return obj


def build(jobs: int | None = None, force: bool = False, verbose: bool = False) -> Path:
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force, verbose), srcs))
    for old in set(OUT_DIR.glob("*.o")) - set(objs):   # objects of earlier source versions
        old.unlink()
    stamp =hashlib.sha256("".join(str(o) for o in objs).encode()).hexdigest()[:16]
    stamp_file = OUT_DIR / "lib.stamp"
    if LIB.exists() and not force and stamp_file.exists() and stamp_file.read_text() == stamp:
        return LIB
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    stamp_file.write_text(stamp)
    return LIB


AOT_DIR = HERE / "bgtq" / "aot"
GOLDEN = HERE.parent / "tests" / "golden"


def prebuild_sets():
    """(name, [(config, table) per head], query rows per head) of the heads the benches and the
    model path attend: the config-4 tables on 3 KV heads (GQA 3), every layer of the
    reference's SmolLM2 calibration (3 KV heads, GQA 3) and of the Qwen calibration (2 KV
    heads, GQA 7)."""
    import numpy as np
    sys.path.insert(0, str(HERE))
    import bgtq
    out = []
    z = np.load(GOLDEN / "config4.npz")
    ct = bgtq.tables(bgtq.BlockGTQParameters.from_arrays(z))
    out.append(("config4", [ct] * 3, 3))
    for fam, heads, rows in (("smollm2", 3, 3), ("qwen", 2, 7)):
        c = np.load(GOLDEN / f"{fam}_calibration.npz")
        tabs = [bgtq.build_tables(c["widths"][i].astype(np.int64), pair_order=c["pair_order"][i].astype(np.int64),
                                  rotation_threshold=int(c["rotation_threshold"]), row_pad=int(c["row_pad"][i]),
                                  norm_stride=int(c["norm_stride"][i])) for i in range(len(c["widths"]))]
        for layer in range(len(tabs) // heads):
            out.append((f"{fam}-layer{layer}", tabs[layer * heads:(layer + 1) * heads], rows))
    return out


def prebuild(jobs: int | None = None) -> list[str]:
    """Compile the layout-specialised decode-attention kernels of prebuild_sets() ahead of time
    into bgtq/aot/ (bgtq_layout_jit_prebuild; files of earlier sources are removed), so that
    launches on a host without nvcc still find them."""
    import ctypes as C
    import numpy as np
    if not (GOLDEN / "config4.npz").exists():
        return []
    lib = C.CDLL(str(LIB))
    AOT_DIR.mkdir(parents=True, exist_ok=True)

    def one(item):
        name, heads, rows = item
        cfgs = [np.ascontiguousarray(c, np.uint32) for c, _ in heads]
        tabs = [np.ascontiguousarray(t, np.float32) for _, t in heads]
        n = len(heads)
        cp = (C.c_void_p * n)(*[a.ctypes.data for a in cfgs])
        tp = (C.c_void_p * n)(*[a.ctypes.data for a in tabs])
        nc = (C.c_size_t * n)(*[a.size for a in cfgs])
        nt = (C.c_size_t * n)(*[a.size for a in tabs])
        buf = C.create_string_buffer(64)
        rc = lib.bgtq_layout_jit_prebuild(str(AOT_DIR).encode(), n, cp, nc, tp, nt, rows, 0, buf, 64)
        if rc != 0:
            lib.bgtq_last_error.restype = C.c_char_p
            raise RuntimeError(f"prebuild {name}: {lib.bgtq_last_error().decode()}")
        return buf.value.decode()

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        names = list(ex.map(one, prebuild_sets()))
    keep = set(names)
    for f in AOT_DIR.glob("*.cubin"):
        if f.name not in keep:
            f.unlink()
    return sorted(keep)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="keep ptxas -v reports in _build/")
    ap.add_argument("--no-prebuild", action="store_true", help="skip the ahead-of-time attention kernels")
    args = ap.parse_args()
    print(build(args.jobs, args.force, args.verbose))
    if not args.no_prebuild:
        print(f"{len(prebuild(args.jobs))} prebuilt attention kernels in {AOT_DIR}")


if __name__ == "__main__":
    sys.exit(main())
