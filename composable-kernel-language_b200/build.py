"""Build libckl_b200.so (runtime, planner and the sm_100a kernel library) in-tree.

    python composable-kernel-language_b200/build.py [--force] [--jobs N]

Every translation unit is compiled by nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); the CUDA runtime is linked statically so the
library loads on hosts without a GPU driver (planning and the C ABI work there).  Objects are
rebuilt when a source or header is newer than they are.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
BUILD = HERE / "_build"
OUTPUT = HERE / "python" / "ckl" / "libckl_b200.so"
TEST_KERNELS = ROOT / "tests" / "native" / "kernels.cu"
TEST_CUBIN = ROOT / "tests" / "native" / "runtime_kernels.cubin"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the B200 build needs the CUDA 12.9 toolkit")
    return found


def sources() -> list[Path]:
    return sorted(p for p in CSRC.rglob("*") if p.suffix in (".cu", ".cpp"))


def headers() -> list[Path]:
    return sorted(p for p in list(CSRC.rglob("*")) + list(INCLUDE.rglob("*"))
                  if p.suffix in (".h", ".hpp", ".cuh"))


def stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def compile_one(source: Path, force: bool) -> Path:
    obj = BUILD / (source.relative_to(CSRC).as_posix().replace("/", "_") + ".o")
    if force or stale(obj, [source, *headers(), Path(__file__)]):
        command = [nvcc(), *ARCH, *FLAGS, "-c", str(source), "-o", str(obj)]
        if source.suffix == ".cpp":
            command[1:1] = ["-x", "cu"]
        result = subprocess.run(command, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    units = sources()
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(lambda s: compile_one(s, force), units))
    if force or stale(OUTPUT, objects):
        command = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(OUTPUT), *map(str, objects),
                   "-cudart", "static", "-lrt", "-lpthread", "-ldl"]
        result = subprocess.run(command, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"link failed:\n{result.stderr}")
    if TEST_KERNELS.exists() and (force or stale(TEST_CUBIN, [TEST_KERNELS])):
        command = [nvcc(), "-cubin", *ARCH, "-O3", str(TEST_KERNELS), "-o", str(TEST_CUBIN)]
        result = subprocess.run(command, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"test CUBIN build failed:\n{result.stderr}")
    return OUTPUT


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int)
    args = parser.parse_args()
    print(build(args.force, args.jobs))
    return 0


if __name__ == "__main__":
    sys.exit(main())
