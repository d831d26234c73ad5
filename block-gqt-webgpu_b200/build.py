"""Build libbgtq.so in-tree for sm_100a with nvcc (no torch extension machinery).

    python block-gqt-webgpu_b200/build.py [--jobs N] [--force]

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
STRICT_FP = {"encode.cu", "rows.cu"}


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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="keep ptxas -v reports in _build/")
    args = ap.parse_args()
    print(build(args.jobs, args.force, args.verbose))


if __name__ == "__main__":
    sys.exit(main())
