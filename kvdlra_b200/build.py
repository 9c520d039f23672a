"""Build the sm_100a CUDA library ``kvdlra_b200/_lib/libkvdlra_b200.so`` in tree.

``python -m kvdlra_b200.build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` with nvcc for ``compute_100a``/``sm_100a`` and links one shared
library with a plain C ABI (``include/kvdlra_b200.h``).  Objects are cached
under ``kvdlra_b200/_lib/obj`` and rebuilt when a source or header changes.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB_DIR = PKG / "_lib"
OBJ_DIR = LIB_DIR / "obj"
LIB = LIB_DIR / "libkvdlra_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-DKVD_BUILD",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the kvdlra_b200 CUDA library cannot be built")


def _digest(src: Path) -> str:
    h = hashlib.sha256()
    for p in sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + [src]:
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def _compile(nvcc: str, src: Path, verbose: bool) -> Path:
    obj = OBJ_DIR / f"{src.stem}.{_digest(src)}.o"
    if obj.exists():
        return obj
    for stale in OBJ_DIR.glob(f"{src.stem}.*.o"):
        stale.unlink()
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    """Compile all sources (in parallel) and link the shared library."""
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose), sources))
    stamp = hashlib.sha256("".join(o.name for o in objs).encode()).hexdigest()[:16]
    stamp_file = LIB_DIR / "libkvdlra_b200.stamp"
    if LIB.exists() and stamp_file.exists() and stamp_file.read_text() == stamp:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    tmp.replace(LIB)
    stamp_file.write_text(stamp)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
