"""Ahead-of-time build of the sm_100a kernel library ``libmak_kvcache.so``.

The reference JIT-compiles its MUSA sources with ``mcc`` into a per-user cache
(musa_aiter/jit/core.py:31-95).  Here the CUDA sources under ``csrc/`` are
compiled once with ``nvcc -gencode arch=compute_100a,code=sm_100a`` into the
package's ``lib/`` folder, so the library travels with the source tree and no
GPU is needed to build it (nvcc cross-compiles).
"""

from __future__ import annotations

import concurrent.futures
import hashlib
import os
import shutil
import subprocess
from dataclasses import dataclass
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
SOURCE_ROOT = PACKAGE_DIR.parent  # musa-aiter_b200/
REPO_ROOT = SOURCE_ROOT.parent
CSRC_DIR = SOURCE_ROOT / "csrc"
INCLUDE_DIR = REPO_ROOT / "include"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_NAME = "libmak_kvcache.so"
LIB_PATH = LIB_DIR / LIB_NAME
BUILD_DIR = SOURCE_ROOT / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


@dataclass(frozen=True)
class BuildResult:
    ok: bool
    message: str
    library_path: Path | None


def _nvcc() -> str | None:
    cand = os.environ.get("NVCC")
    if cand and Path(cand).exists():
        return cand
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    return str(default) if default.exists() else None


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _fingerprint() -> str:
    h = hashlib.sha256()
    for path in sources() + sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h")):
        h.update(path.name.encode())
        h.update(path.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()


def _stamp_path() -> Path:
    return LIB_DIR / (LIB_NAME + ".stamp")


def is_built() -> bool:
    return LIB_PATH.exists() and _stamp_path().exists() and _stamp_path().read_text().strip() == _fingerprint()


def build(force: bool = False, verbose: bool = False) -> BuildResult:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``lib/libmak_kvcache.so``."""
    if not force and is_built():
        return BuildResult(True, "up to date", LIB_PATH)
    nvcc = _nvcc()
    if nvcc is None:
        return BuildResult(False, "nvcc compiler not found", None)
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    include = ["-I", str(INCLUDE_DIR), "-I", str(CSRC_DIR)]

    def compile_one(src: Path) -> tuple[Path, subprocess.CompletedProcess]:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *include, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        return obj, subprocess.run(cmd, capture_output=True, text=True)

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        results = list(pool.map(compile_one, sources()))
    errors = [proc.stderr for _, proc in results if proc.returncode != 0]
    if errors:
        return BuildResult(False, "\n".join(errors), None)
    tmp = LIB_DIR / (LIB_NAME + ".tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *[str(obj) for obj, _ in results]]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        return BuildResult(False, proc.stderr, None)
    os.replace(tmp, LIB_PATH)
    _stamp_path().write_text(_fingerprint() + "\n")
    return BuildResult(True, "built", LIB_PATH)


if __name__ == "__main__":  # pragma: no cover - manual entry point
    result = build(force=True, verbose=True)
    print(result.message)
    raise SystemExit(0 if result.ok else 1)
