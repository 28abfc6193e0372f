"""Builds libmg_b200.so, the C-ABI library behind include/mg_b200.h.

Every .cu under csrc/ is compiled for sm_100a only, in parallel, and linked
into one shared library with the CUDA runtime linked statically, so the
library carries its own runtime and needs nothing from the Python side but a
stream handle. preprocess_fwd.cu is compiled without multiply-add contraction
(-fmad=false): its outputs feed the binning decisions and are required to be
bit-identical to the CPU restatement in oracle/.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_native"
LIB = OUT_DIR / "libmg_b200.so"
OBJ_DIR = ROOT / "_build" / "mg_b200"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                 "-Xptxas", "-warn-spills", "-I", str(ROOT / "include")]
PER_FILE = {"preprocess_fwd.cu": ["-fmad=false"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmg_b200.so")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "mg_b200.h",
                                                      Path(__file__)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in _deps())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile and link; returns the library path. No-op when up to date."""
    if not force and up_to_date():
        return LIB
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    extra = list(extra or [])

    def compile_one(src: Path) -> Path:
        obj = OBJ_DIR / (src.stem + ".o")
        cmd = [cc, *COMMON, *PER_FILE.get(src.name, []), *extra, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{r.stdout}{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(f"[{src.name}]\n{r.stdout}{r.stderr}", file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
           "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
