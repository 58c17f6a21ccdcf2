"""Builds libkush_sm100.so, the sm_100a kernel library, in-tree with nvcc (cross-compiles without a GPU).

    python -m kushkash_b200.build            # or kushkash_b200.build.build()

Every .cu under csrc/ is compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`), in parallel, then
linked into kushkash_b200/libkush_sm100.so with the CUDA runtime linked statically (the library needs only the
NVIDIA driver at run time).  A rebuild happens when any source or header is newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libkush_sm100.so"
OBJ = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (CUDA toolkit required to build kushkash_b200)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile (if stale) and return the library path.  `extra` adds nvcc flags (e.g. ["-Xptxas", "-v"])."""
    if not force and not extra and not _stale():
        return LIB
    OBJ.mkdir(exist_ok=True)
    cc = nvcc()
    flags = NVCC_FLAGS + ARCH + list(extra or [])

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = OBJ / (src.stem + ".o")
        cmd = [cc, *flags, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr[-6000:]}")
        return obj, r.stderr

    with ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        results = list(ex.map(compile_one, sources()))
    for obj, log in results:
        if verbose and log.strip():
            print(f"--- {obj.name}\n{log}", file=sys.stderr)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp)] + [str(o) for o, _ in results]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stderr[-6000:]}")
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    print(build(force=True, verbose=v, extra=["-Xptxas", "-v"] if v else None))
