"""Build libflow2surf_sm100.so from csrc/*.cu with nvcc for sm_100a.

Objects go to _build/ beside this file; the shared library lands inside the
Python package (flow2surf_b200/libflow2surf_sm100.so) so that it travels with
the source tree. Only sources newer than their object (or than any header) are
recompiled.

    python jittor-flow2surf_b200/build.py [--force] [--jobs N]
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
LIBRARY = HERE / "flow2surf_b200" / "libflow2surf_sm100.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-warn-spills",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required")
    return path


def _newest_header() -> float:
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in headers), default=0.0)


def _compile(src: Path, force: bool, extra: list[str]) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if not force and obj.exists():
        if obj.stat().st_mtime >= max(src.stat().st_mtime, _newest_header()):
            return obj, ""
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False,
          extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=jobs) as pool:
        results = list(pool.map(lambda s: _compile(s, force, extra or []), sources))
    objects = [obj for obj, _ in results]
    if verbose:
        for _, log in results:
            if log.strip():
                print(log, file=sys.stderr)
    newest = max(o.stat().st_mtime for o in objects)
    if force or not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objects),
               "-o", str(LIBRARY)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--verbose", action="store_true", help="print ptxas output")
    parser.add_argument("--ptxas-info", action="store_true", help="add -Xptxas -v")
    args = parser.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    lib = build(force=args.force or args.ptxas_info, jobs=args.jobs,
                verbose=args.verbose or args.ptxas_info, extra=extra)
    print(lib)


if __name__ == "__main__":
    main()
