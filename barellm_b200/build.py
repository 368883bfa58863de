"""Builds the sm_100a C-ABI library ``barellm_b200/_lib/libbarellm_b200.so``.

The library is compiled in-tree with ``nvcc`` (it cross-compiles without a
GPU), one object per ``csrc/*.cu`` file in parallel, then linked with the CUDA
runtime statically so the library needs only the driver at run time.

    python -m barellm_b200.build [--force] [--verbose-ptxas]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "_lib"
OBJ_DIR = PKG / "_build"
LIB_NAME = "libbarellm_b200.so"
LIB_PATH = OUT_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "--use_fast_math",
    "-I",
    str(INCLUDE),
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the barellm_b200 CUDA library cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _needs_rebuild(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose_ptxas: bool) -> str:
    cmd = [nvcc_path(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> Path:
    """Compiles every csrc/*.cu for sm_100a and links the shared library."""
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    hdrs = headers()
    jobs = []
    for src in sources():
        obj = OBJ_DIR / (src.stem + ".o")
        if force or verbose_ptxas or _needs_rebuild(obj, [src, *hdrs]):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, verbose_ptxas): s for s, o in jobs}
            for fut in cf.as_completed(futs):
                log = fut.result()
                if log and (verbose_ptxas or not quiet):
                    print(f"== {futs[fut].name}\n{log}", file=sys.stderr)
    objs = [OBJ_DIR / (s.stem + ".o") for s in sources()]
    if force or jobs or _needs_rebuild(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, verbose_ptxas=args.verbose_ptxas, quiet=False)
    print(path)


if __name__ == "__main__":
    main()
