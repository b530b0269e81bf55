"""Builds libqwen36_paged_kv.so, the sm_100a kernels behind include/qwen36_paged_kv.h.

The library is compiled in-tree (``<package>/lib/``) with nvcc for ``sm_100a`` only, links the
CUDA runtime statically and has no torch dependency, so any FFI can load it. Object files are
compiled in parallel and relinked only when a source or header is newer than the library.

    python qwen3.6-2080ti_b200/build_native.py [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
BUILD_DIR = PACKAGE_DIR / "_build"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_NAME = "libqwen36_paged_kv.so"
SOURCES = ("pkv_capi.cu", "pkv_pages.cu", "pkv_decode.cu", "pkv_prefill.cu", "pkv_rope.cu", "pkv_oproj.cu")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
NVCC_FLAGS = (
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
)


def nvcc_path() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def library_path() -> Path:
    return LIB_DIR / LIB_NAME


def _inputs_mtime() -> float:
    files = [CSRC / name for name in SOURCES] + list(CSRC.glob("*.cuh")) + list((REPO_ROOT / "include").glob("*.h"))
    files.append(Path(__file__))
    return max(path.stat().st_mtime for path in files)


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(REPO_ROOT / "include"), "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        print(" ".join(cmd))
    return proc.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library if needed and returns its path."""
    lib = library_path()
    if not force and lib.exists() and lib.stat().st_mtime >= _inputs_mtime():
        return lib
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objects = [BUILD_DIR / (Path(name).stem + ".o") for name in SOURCES]
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        futures = [pool.submit(_compile, CSRC / name, obj, verbose) for name, obj in zip(SOURCES, objects)]
        logs = [future.result() for future in futures]
    (BUILD_DIR / "ptxas.log").write_text("\n".join(logs))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, lib)
    return lib


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
