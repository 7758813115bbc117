"""Build libhlm_b200.so from csrc/ for sm_100a (in-tree, no JIT cache).

    python -m hackable_lm_b200.build            # incremental
    python -m hackable_lm_b200.build --force    # rebuild everything

Each .cu is compiled to an object under _build/ (in parallel), then linked
into hackable_lm_b200/libhlm_b200.so next to this file.  nvcc cross-compiles
for sm_100a, so this works on a machine without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
BUILD_DIR = PKG_DIR.parent / "_build"
LIB_NAME = "libhlm_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool) -> tuple[Path, str]:
    cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stdout + proc.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libhlm_b200.so; return its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    sources = _sources()
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        stale = (
            force
            or not obj.exists()
            or obj.stat().st_mtime < src.stat().st_mtime
            or obj.stat().st_mtime < newest_header
        )
        if stale:
            jobs.append((src, obj))
    logs = []
    if jobs:
        workers = min(len(jobs), max(1, os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(max_workers=workers) as pool:
            futs = [pool.submit(_compile, nvcc, s, o, verbose) for s, o in jobs]
            for f in futs:
                logs.append(f.result()[1])
    relink = bool(jobs) or not LIB_PATH.exists() or any(
        o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objs
    )
    if relink:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        # Shared cudart: the library then uses the same runtime instance (current
        # device, streams) as the PyTorch process that loads it.
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "shared",
               "-Xlinker", "-rpath,/usr/local/cuda/lib64", "-o", str(tmp), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    if verbose:
        for log in logs:
            sys.stdout.write(log)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill info")
    args = ap.parse_args()
    path = build(force=args.force, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main()
