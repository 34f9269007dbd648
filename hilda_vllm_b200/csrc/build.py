"""Builds libhilda_b200.so (all CUDA kernels + the C ABI) in-tree for sm_100a with nvcc.

Usage: python -m hilda_vllm_b200.csrc.build [--force] [--verbose]
The library lands next to the package's __init__.py so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
BUILD_DIR = ROOT / "_build"
LIB_NAME = "libhilda_b200.so"
LIB_PATH = PKG / LIB_NAME

SOURCES = [
    "abi.cu",
    "store_kv.cu",
    "paged_decode.cu",
    "paged_decode_tc.cu",
    "prefill_tc.cu",
    "pack_decode.cu",
    "layer_ops.cu",
    "allreduce.cu",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda_home) / "bin" / "nvcc"
    if path.exists():
        return str(path)
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh"))
    files += sorted(INCLUDE.glob("*.h"))
    files.append(Path(__file__))
    return files


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    lib_m = LIB_PATH.stat().st_mtime
    return all(f.stat().st_mtime <= lib_m for f in _inputs())


def _compile(nvcc: str, src: Path, obj: Path, extra: list[str], verbose: bool) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr, flush=True)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile every kernel source for sm_100a and link the shared library."""
    if not force and up_to_date():
        return LIB_PATH
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    extra = list(extra_flags or [])
    objs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        futs = []
        for s in SOURCES:
            obj = BUILD_DIR / (Path(s).stem + ".o")
            objs.append(obj)
            futs.append(ex.submit(_compile, nvcc, CSRC / s, obj, extra, verbose))
        for f in futs:
            f.result()
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers / spills per kernel")
    args = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_verbose else []
    path = build(force=args.force or args.ptxas_verbose, verbose=args.verbose or args.ptxas_verbose, extra_flags=extra)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
