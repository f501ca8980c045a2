"""Build ``mambaqc_b200/libmambaqc_b200.so`` from the CUDA/C++ sources in this folder.

Plain nvcc, in-tree, for sm_100a only:

    python -m mambaqc_b200.csrc.build            # incremental
    python -m mambaqc_b200.csrc.build --force    # rebuild everything
    MQC_PTXAS_VERBOSE=1 python -m mambaqc_b200.csrc.build --force   # -Xptxas -v

The library has a pure C ABI (``include/mambaqc_b200.h``) and links the CUDA
runtime statically, so it carries no torch dependency; the Python package loads
it with ctypes.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
BUILD_DIR = PKG / "_build"
LIB = PKG / "libmambaqc_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden", "-Xfatbin", "-compress-all"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def _sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def _headers() -> list[Path]:
    return sorted([*CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")])


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD_DIR / (src.name + ".o")
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stdout + proc.stderr


def build(force: bool = False, jobs: int | None = None, quiet: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    verbose_ptxas = os.environ.get("MQC_PTXAS_VERBOSE") == "1"
    todo = []
    for s in srcs:
        obj = BUILD_DIR / (s.name + ".o")
        if (force or verbose_ptxas or not obj.exists()
                or obj.stat().st_mtime < max(s.stat().st_mtime, newest_header)):
            todo.append(s)
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj, log in ex.map(lambda s: _compile(s, verbose_ptxas), todo):
            if log.strip() and (verbose_ptxas or not quiet):
                print(f"[{obj.name}]\n{log}", file=sys.stderr)
    objs = [BUILD_DIR / (s.name + ".o") for s in srcs]
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB)
        if not quiet:
            print(f"built {LIB}", file=sys.stderr)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    args = ap.parse_args()
    build(force=args.force, jobs=args.jobs)


if __name__ == "__main__":
    main()
