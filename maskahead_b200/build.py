"""Build the sm_100a shared library ``maskahead_b200/_lib/libmaskahead_b200.so``.

    python -m maskahead_b200.build            # compile what changed
    python -m maskahead_b200.build --force    # recompile everything

Each ``csrc/*.cu`` compiles to an object with nvcc (``-gencode arch=compute_100a,
code=sm_100a``), the objects link into one shared library with the CUDA runtime linked
statically, so the library depends on nothing but the driver. It exports only the C ABI
of ``include/maskahead_b200.h``.
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
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libmaskahead_b200.so"
BUILD = ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", str(ROOT / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the maskahead_b200 kernels need the CUDA toolkit to build")


def _newest_header() -> float:
    hdrs = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hdrs), default=0.0)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if any source is newer than it; return its path."""
    sources = sorted(CSRC.glob("*.cu"))
    BUILD.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    hdr_time = _newest_header()
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
            cmd = [cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
            if verbose and res.stderr:
                sys.stderr.write(res.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(compile_one, sources))
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest_obj:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="pass -Xptxas -v (registers, spills)")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
