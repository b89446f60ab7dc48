"""Build the sm_100a C-ABI library in-tree.

    python pic-kvcache_b200/build.py [--force] [--debug]

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` (``-gencode
arch=compute_100a,code=sm_100a -lineinfo``) into
``cacheblend_b200/_lib/libcacheblend_b200.so``.  The CUDA runtime is linked
statically and the driver library is not linked, so the shared object loads
(and its exported symbols can be checked) on a machine without a GPU.  The
build is incremental: it is skipped when the library is newer than every
source and header.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_DIR = PKG_ROOT / "cacheblend_b200" / "_lib"
LIB_PATH = LIB_DIR / "libcacheblend_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs() -> list[Path]:
    return (sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
            + [Path(__file__)])


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    built = LIB_PATH.stat().st_mtime
    return all(path.stat().st_mtime <= built for path in _inputs())


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    if not force and not debug and up_to_date():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = PKG_ROOT / "_build"
    obj_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    common = [
        "-std=c++17",
        "-O3",
        *ARCH_FLAGS,
        "-lineinfo",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "-I",
        str(INCLUDE),
        "-I",
        str(CSRC),
        "--expt-relaxed-constexpr",
    ]
    if debug:
        common.append("-DCB_DEBUG=1")
    if verbose:
        common += ["-Xptxas", "-v"]
    objects = []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *common, "-c", str(src), "-o", str(obj)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
        if verbose and proc.stderr:
            print(proc.stderr, file=sys.stderr)
        objects.append(str(obj))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *objects]
    proc = subprocess.run(link, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--debug", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print -Xptxas -v resource usage")
    args = parser.parse_args()
    path = build(force=args.force, debug=args.debug, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main()
