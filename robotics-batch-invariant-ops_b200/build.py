"""Build the sm_100a kernel library in-tree.

Compiles every ``csrc/*.cu`` translation unit with nvcc for
``arch=compute_100a,code=sm_100a`` and links them into
``batch_invariant_ops/libbio_sm100.so`` (C ABI declared in
``include/bio_sm100.h``).  Objects go to ``_build/`` next to this file.

Usage::

    python build.py [--verbose-ptxas] [--jobs N]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
OUTPUT = HERE / "batch_invariant_ops" / "libbio_sm100.so"
INCLUDE = HERE.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{INCLUDE}",
]


def _nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the sm_100a kernel library cannot be built")
    return path


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers_mtime() -> float:
    return max(p.stat().st_mtime for p in [*CSRC.glob("*.cuh"), *INCLUDE.glob("*.h"), Path(__file__)])


def _compile(src: Path, verbose_ptxas: bool, incremental: bool = False) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if (incremental and obj.exists()
            and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime())):
        return obj, ""
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def _needs_rebuild() -> bool:
    if not OUTPUT.exists():
        return True
    newest = max(
        p.stat().st_mtime
        for p in [*CSRC.glob("*.cu"), *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h"), Path(__file__)]
    )
    return OUTPUT.stat().st_mtime < newest


def build(verbose_ptxas: bool = False, jobs: int | None = None, force: bool = False) -> Path:
    """Compile and link the library; returns the path of the shared object."""
    if not force and not _needs_rebuild():
        return OUTPUT
    BUILD.mkdir(exist_ok=True)
    sources = _sources()
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    logs = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        # unforced builds recompile only the units older than their source or
        # any header; a forced build recompiles everything
        results = list(pool.map(lambda s: _compile(s, verbose_ptxas, not force), sources))
    objs = [obj for obj, _ in results]
    logs = [log for _, log in results if log.strip()]
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, OUTPUT)
    if verbose_ptxas:
        for log in logs:
            sys.stderr.write(log)
    return OUTPUT


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose-ptxas", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    out = build(args.verbose_ptxas, args.jobs, force=args.force or args.verbose_ptxas)
    print(out)


if __name__ == "__main__":
    main()
