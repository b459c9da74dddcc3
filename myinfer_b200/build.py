"""Build libm5cuda.so (the sm_100a kernels + C ABI) in place with nvcc.

Usage: ``python -m myinfer_b200.build [--verbose]``.  Every ``csrc/*.cu`` is
compiled for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``),
without fast-math (the KV quantizer must round exactly like the CPU rule),
and linked into ``myinfer_b200/libm5cuda.so`` next to this file.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB = HERE / "libm5cuda.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def nccl_paths():
    """Include and library directories of the NCCL that ships with torch."""
    try:
        import nvidia.nccl as nccl  # type: ignore
        base = Path(list(nccl.__path__)[0])
        if (base / "include" / "nccl.h").exists():
            return base / "include", base / "lib"
    except Exception:
        pass
    return None, None


def _compile(src: Path, verbose: bool) -> Path:
    out = OBJ / (src.stem + ".o")
    deps = [src] + list(CSRC.glob("*.cuh")) + [INCLUDE / "m5cuda.h"]
    if out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return out
    inc, _ = nccl_paths()
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-c", str(src), "-o", str(out),
           f"-I{INCLUDE}", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]
    if inc is not None:
        cmd += [f"-I{inc}", "-DM5_HAVE_NCCL=1"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    return out


def build(verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if LIB.exists() and all(LIB.stat().st_mtime >= o.stat().st_mtime for o in objs):
        return LIB
    _, libdir = nccl_paths()
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs)]
    if libdir is not None:
        cmd += [f"-L{libdir}", "-l:libnccl.so.2", "-Xlinker", f"-rpath={libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv))
