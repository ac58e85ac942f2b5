"""Build the tideway_b200 CUDA library for sm_100a (B200) in-tree.

    python -m tideway_b200.build            # incremental
    python -m tideway_b200.build --force    # rebuild everything

Every ``csrc/*.cu`` is compiled with nvcc for ``sm_100a`` only and linked into
``tideway_b200/_lib/libtideway_b200.so`` (CUDA runtime linked statically, so the library
only needs the driver).  Objects go to ``_build/`` at the repository root.
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
BUILD = ROOT / "_build"
LIB = PKG / "_lib" / "libtideway_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the tideway_b200 CUDA library cannot be built")


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None,
          lib: Path = LIB, build_dir: Path = BUILD) -> Path:
    """Compile and link; ``lib``/``build_dir`` redirect the outputs (tuning builds)."""
    lib, build_dir = Path(lib), Path(build_dir)
    build_dir.mkdir(parents=True, exist_ok=True)
    lib.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    flags = NVCC_FLAGS + list(extra_flags or [])
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = build_dir / (src.stem + ".o")
        if force or _stale(obj, src):
            cmd = [cc, *flags, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
            if verbose and res.stderr:
                print(res.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources))
    if force or not lib.exists() or any(o.stat().st_mtime > lib.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(lib), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_info else []
    out = build(force=a.force or a.ptxas_info, verbose=a.verbose or a.ptxas_info, extra_flags=extra)
    print(out)


if __name__ == "__main__":
    sys.exit(main())
