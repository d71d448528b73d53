"""Build the sm_100a shared library ``libda_b200.so`` next to this file.

Every ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` and linked
into one shared library exporting the C ABI declared in
``include/da_b200.h``.  Object files go to ``_build/`` at the repository
root; a file is recompiled only when it or a header changed.

Usage: ``python -m double_attention_b200.build [--force] [-j N]``.
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
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build"
LIB_PATH = PACKAGE_DIR / "libda_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the sm_100a library cannot be built")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _needs_build(src: Path, obj: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    mtime = obj.stat().st_mtime
    return src.stat().st_mtime > mtime or newest_header > mtime


def _compile(nvcc: str, src: Path, obj: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return src, proc.stdout + proc.stderr


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> Path:
    """Compile (incrementally) and link the library; returns its path."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError("no CUDA sources found")
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objects = [BUILD_DIR / (src.stem + ".o") for src in sources]
    todo = [(s, o) for s, o in zip(sources, objects) if force or _needs_build(s, o, newest_header)]
    logs: list[str] = []
    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
            for src, log in pool.map(lambda so: _compile(nvcc, so[0], so[1], verbose_ptxas), todo):
                if log.strip():
                    logs.append(f"== {src.name}\n{log}")
    relink = force or bool(todo) or not LIB_PATH.exists()
    if not relink:
        lib_mtime = LIB_PATH.stat().st_mtime
        relink = any(o.stat().st_mtime > lib_mtime for o in objects)
    if relink:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    if verbose_ptxas and logs:
        print("\n".join(logs))
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("-j", "--jobs", type=int, default=None)
    parser.add_argument("--ptxas-verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose_ptxas=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
