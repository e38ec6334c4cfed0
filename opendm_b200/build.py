"""Build the sm_100a CUDA library ``libopendm_muon.so`` in-tree.

Compiles every ``csrc/*.cu`` file with nvcc for ``sm_100a`` (objects in
parallel), links them into ``opendm_b200/libopendm_muon.so`` and skips the work
when the library is newer than every source and header. The CUDA runtime is
linked statically, so the library needs only the NVIDIA driver at run time.

    python -m opendm_b200.build [--force] [--debug]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_NAME = "libopendm_muon.so"
LIB_PATH = PKG / LIB_NAME
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    """Compile the library if needed and return its path."""
    if not force and not is_stale():
        return LIB_PATH
    nvcc = _nvcc()
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    common = [nvcc, *ARCH_FLAGS, "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
              "-O0" if debug else "-O3"]
    if debug:
        common.append("-DMUON_DEBUG=1")

    def compile_one(src: Path) -> Path:
        obj = objdir / (src.stem + ".o")
        cmd = common + ["-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, debug=args.debug, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main(sys.argv[1:])
