"""Build libdh_b200.so (all CUDA kernels, sm_100a) in-tree.

``python -m diffusionhard_b200.build`` compiles every ``csrc/*.cu`` with nvcc
for ``arch=compute_100a,code=sm_100a`` and links them into
``diffusionhard_b200/lib/libdh_b200.so``.  Objects are rebuilt only when a
source or header is newer than the object.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = PKG / "lib" / "obj"
LIB_PATH = LIB_DIR / "libdh_b200.so"
INCLUDE = PKG.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-rdc=true",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
    "--expt-relaxed-constexpr",
    "-I", str(CSRC), "-I", str(INCLUDE),
]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libdh_b200.so")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    nvcc = _nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    deps = _headers()
    flags = NVCC_FLAGS + list(extra_flags or [])
    jobs = []
    for src in sources:
        obj = OBJ_DIR / (src.stem + ".o")
        if _stale(obj, src, deps):
            jobs.append([nvcc, *flags, "-c", str(src), "-o", str(obj)])

    def run(cmd: list[str]) -> None:
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
        if verbose and proc.stderr.strip():
            print(proc.stderr, file=sys.stderr)

    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        list(pool.map(run, jobs))
    objs = [OBJ_DIR / (s.stem + ".o") for s in sources]
    if jobs or not LIB_PATH.exists() or any(o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        run([nvcc, "-shared", "-rdc=true", "-gencode", "arch=compute_100a,code=sm_100a",
             "-o", str(tmp), *map(str, objs), "-lcuda"])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_oracle(reference_root: str | None = None) -> None:
    """Build the CPU checkers in oracle/ (test infrastructure).  The reference
    C++ checkers are compiled from the reference tree given as an argument or
    by $DH_REFERENCE_ROOT, else from its checkout at /root/reference when that
    exists; without a tree only the plain-C oracle is built."""
    oracle_dir = PKG.parent / "oracle"
    subprocess.run(["make", "-s", "-C", str(oracle_dir)], check=True)
    ref = Path(reference_root or os.environ.get("DH_REFERENCE_ROOT") or "/root/reference")
    if (ref / "hls").is_dir():
        subprocess.run(["make", "-s", "-C", str(oracle_dir), "ref", f"REF={ref}"], check=True)


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
