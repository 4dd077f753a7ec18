"""Build libpkv.so (the sm_100a kernels behind include/pkv.h) in-tree.

The library is compiled with nvcc straight to sm_100a machine code, links the
CUDA runtime statically and exports only the ``pkv_*`` C entry points (a
linker version script hides everything else, so the runtime inside the
library never interposes on the one PyTorch loads). Run as
``python grpo_training_engine_b200/build.py`` or through
``__graft_entry__.build()``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_PATH = PKG_DIR / "libpkv.so"

SOURCES = ["pkv_copy.cu", "pkv_decode.cu", "pkv_noalloc.cu", "pkv_sample.cu", "pkv_glue.cu", "pkv_linear.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda_home) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile libpkv.so if any source or header is newer than it: each source
    to an object in parallel, then one link."""
    from concurrent.futures import ThreadPoolExecutor

    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [INCLUDE / "pkv.h"]
    if not force and not _stale(LIB_PATH, deps):
        return LIB_PATH
    vscript = CSRC / "pkv.map"
    tmp = LIB_PATH.with_suffix(".so.tmp")
    common = [_nvcc(), "-O3", "-std=c++17", *ARCH_FLAGS, "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE)]
    objdir = PKG_DIR / "_build"
    objdir.mkdir(exist_ok=True)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")

    objs = [objdir / (Path(s).stem + ".o") for s in SOURCES]
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        list(pool.map(run, [common + ["-c", str(CSRC / s), "-o", str(o)] for s, o in zip(SOURCES, objs)]))
    run([*common, "-shared", "-Xlinker", f"--version-script={vscript}", "-o", str(tmp), *map(str, objs)])
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True))
