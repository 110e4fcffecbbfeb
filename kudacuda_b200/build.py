"""Build the sm_100a C-ABI library in-tree: kudacuda_b200/lib/libkudacuda.so.

Compiles every kudacuda_b200/csrc/*.cu with nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``), links the CUDA runtime
statically so the library has no runtime dependency beyond libc and the
driver (resolved lazily), and writes the result next to the package so it
travels with the source tree.  Objects are rebuilt only when a source or
header is newer than the library.

    python -m kudacuda_b200.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_PATH = LIB_DIR / "libkudacuda.so"
OBJ_DIR = PACKAGE_DIR / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    env = os.environ.get("NVCC")
    if env:
        return env
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    if default.exists():
        return str(default)
    raise FileNotFoundError("nvcc not found (set NVCC or put it on PATH)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs_mtime() -> float:
    files = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return max(f.stat().st_mtime for f in files if f.is_file())


def needs_build() -> bool:
    return not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < _inputs_mtime()


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library; returns its path."""

    if not force and not needs_build():
        return LIB_PATH
    nvcc = nvcc_path()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()

    def compile_one(src: Path) -> Path:
        obj = OBJ_DIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
        if verbose and proc.stderr:
            print(proc.stderr, file=sys.stderr)
        return obj

    workers = jobs or min(len(srcs), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=workers) as pool:
        objs = list(pool.map(compile_one, srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, *ARCH_FLAGS, "-shared", "--cudart=static", "-o", str(tmp), *map(str, objs), "-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(link), flush=True)
    proc = subprocess.run(link, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
