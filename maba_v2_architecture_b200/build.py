"""Builds libmaba_b200.so (the C-ABI library of the sm_100a kernels) in-tree.

Every ``csrc/*.cu`` is compiled with nvcc for ``sm_100a`` into ``_build/`` at the
repository root and linked into ``maba_v2_architecture_b200/libmaba_b200.so``.
The CUDA runtime is linked statically, so the library only needs the driver.
Rebuilds are incremental on file modification times (any header change
rebuilds every object).

    python -m maba_v2_architecture_b200.build [--force] [-j N] [-v]
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
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build"
LIB_NAME = "libmaba_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-DMABA_BUILD_SHARED",
]


def nvcc_path() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o",
           str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stdout + res.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile (if needed) and return the path of libmaba_b200.so."""
    BUILD_DIR.mkdir(exist_ok=True)
    headers = _headers()
    srcs = _sources()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    todo = []
    objs = []
    for src in srcs:
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_verbose or _stale(obj, [src, *headers, Path(__file__)]):
            todo.append((src, obj))
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = [ex.submit(_compile, s, o, verbose, extra) for s, o in todo]
            for f in futs:
                obj, log = f.result()
                if ptxas_verbose and log.strip():
                    print(f"== {obj.name}\n{log}", flush=True)
    if force or todo or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print ptxas register/spill/smem usage")
    args = ap.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose, ptxas_verbose=args.ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
