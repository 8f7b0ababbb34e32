"""Build the sm_100a C-ABI library ``libslm_turbo_b200.so`` in-tree with nvcc.

    python -m slm_turbo_b200.build          # or build_library() from Python

The library is written next to this file so that it travels with the source
tree; there is no JIT cache and no Python extension module.  Flags: sm_100a
only, -O3, -lineinfo, IEEE division/rounding (no --use_fast_math: the
quantizers must match the reference bit for bit).
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
LIB_NAME = "libslm_turbo_b200.so"
LIB_PATH = HERE / LIB_NAME
SOURCES = ["decode.cu", "store.cu", "decode_noalloc.cu",
           "decode_d64_paged.cu", "decode_d64_contig.cu", "decode_d80_paged.cu", "decode_d80_contig.cu",
           "decode_d128_paged.cu", "decode_d128_contig.cu", "prefill.cu"]
HEADERS = ["ptx.cuh", "decode_common.cuh", "decode_kernels.cuh", "decode_dispatch.cuh", "quant_store.cuh",
           "internal.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3",
    "-cudart", "shared",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "slm_turbo_b200.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False, extra_flags=None) -> Path:
    """Compile every .cu source into one shared library (skips if up to date)."""
    if not force and not _stale():
        return LIB_PATH
    build_dir = HERE / "_build"
    build_dir.mkdir(exist_ok=True)
    flags = NVCC_FLAGS + list(extra_flags or [])
    cmds = []
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmds.append(([nvcc(), *flags, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(CSRC / src), "-o", str(obj)],
                     str(obj)))

    def compile_one(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        return subprocess.run(cmd, capture_output=not verbose, text=True)

    # the translation units are independent: compile them in parallel
    with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, [c for c, _ in cmds]))
    for (cmd, _), res in zip(cmds, results):
        if res.returncode != 0:
            sys.stderr.write((res.stdout or "") + (res.stderr or ""))
            raise subprocess.CalledProcessError(res.returncode, cmd, res.stdout, res.stderr)
        if not verbose and extra_flags and res.stderr:
            sys.stderr.write(res.stderr)
    objs = [o for _, o in cmds]
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "shared",
           "-Xlinker", "-rpath,/usr/local/cuda/lib64", *objs, "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    force = "--force" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None
    print(build_library(force=force or bool(extra), verbose=True, extra_flags=extra))
