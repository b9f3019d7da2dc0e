"""Build ``libneurosim_b200.so`` in-tree with nvcc for sm_100a.

The library is plain CUDA C++ behind a C ABI (``include/neurosim_b200.h``):
no PyTorch headers, no JIT cache.  Object files go to ``csrc/_build/``; the
shared library lands next to this file so it ships with the source tree.

    python -m neurosim_gpu_b200.build [--force] [--debug]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
LIBRARY = PACKAGE / "libneurosim_b200.so"
SOURCES = ("tick.cu", "tiled.cu", "pels.cu", "pels_rows.cu", "cluster.cu", "encode.cu", "capi.cu")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libneurosim_b200.so")
    return path


def _flags(debug: bool) -> list[str]:
    flags = ARCH + ["-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                    "-I", str(INCLUDE), "-I", str(CSRC)]
    flags += ["-O0", "-G"] if debug else ["-O3"]
    if os.environ.get("NSB_PTXAS_VERBOSE"):
        flags += ["-Xptxas", "-v"]
    return flags


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in inputs)


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library if any source or header is newer than it."""
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    objdir = CSRC / "_build"
    objdir.mkdir(exist_ok=True)
    compiler = nvcc()
    flags = _flags(debug)
    jobs = []
    for name in SOURCES:
        src = CSRC / name
        obj = objdir / (name + ".o")
        if force or _stale(obj, [src, *headers]):
            jobs.append([compiler, *flags, "-c", str(src), "-o", str(obj)])
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        results = list(pool.map(lambda cmd: subprocess.run(cmd, capture_output=True, text=True),
                                jobs))
    for cmd, result in zip(jobs, results):
        if verbose or result.returncode:
            print(" ".join(cmd))
            print(result.stdout + result.stderr)
        if result.returncode:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}")
    objects = [objdir / (name + ".o") for name in SOURCES]
    if force or jobs or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [compiler, *ARCH, "-shared", "-o", str(tmp), *map(str, objects)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError("link failed:\n" + result.stdout + result.stderr)
        os.replace(tmp, LIBRARY)
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--debug", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, debug=args.debug, verbose=args.verbose))


if __name__ == "__main__":
    main()
