"""Build recipe for libjetspec_b200.so (sm_100a only).

Each CUDA translation unit under csrc/ is compiled with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared library that
sits beside this file, so the built artefact travels with the source tree.
"""
from __future__ import annotations

import concurrent.futures
import os
from pathlib import Path
import shutil
import subprocess

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
LIBRARY = PACKAGE_DIR / "libjetspec_b200.so"
INCLUDE = PACKAGE_DIR.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2",
                "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def nvcc_path() -> str:
    candidates = [shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for candidate in candidates:
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the sm_100a kernels need the CUDA toolkit")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(objects: list[Path]) -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(path.stat().st_mtime > built for path in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libjetspec_b200.so in place."""
    build_dir = PACKAGE_DIR / "_build"
    objects = [build_dir / (src.stem + ".o") for src in sources()]
    if not force and not _stale(objects):
        return LIBRARY
    build_dir.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    extra = ["-Xptxas", "-v"] if verbose else []

    def compile_one(src: Path, obj: Path):
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src),
               "-o", str(obj)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{result.stderr}")
        return result.stderr

    workers = min(len(objects), os.cpu_count() or 1)
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
        logs = list(pool.map(compile_one, sources(), objects))
    if verbose:
        for log in logs:
            print(log)
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
