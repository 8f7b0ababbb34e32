"""Compile the REFERENCE's own CUDA extension into ``oracle/_ref/`` (checker only).

    python -m oracle.build_ref /path/to/slm-turbo
    SLMT_REFERENCE_TREE=/path/to/slm-turbo python -m oracle.build_ref

Builds kernels/kv_dequant_cuda.cu (+ kv_dequant_kernels.cuh) of the slm-turbo
tree where it lies, unmodified, for sm_100a, with the same flags its JIT
loader uses (kernels/kv_dequant.py:60-63 with SLM_TURBO_CUDA_ARCH=100a).  The
output is a torch extension module ``slm_turbo_kv_dequant_cuda*.so`` in
``oracle/_ref/`` (git-ignored; it travels to the GPU box with the tree).  It
is used only by tests and golden-vector scripts to pin the CPU oracle against
the reference's CUDA kernels; nothing in the product imports it.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"
EXT_NAME = "slm_turbo_kv_dequant_cuda"


def built_path():
    cands = sorted(REF_DIR.glob(f"{EXT_NAME}*.so"))
    return cands[0] if cands else None


def reference_tree(arg=None):
    """The slm-turbo source tree to build from: the argument, else the
    SLMT_REFERENCE_TREE environment variable; None when neither names an
    existing directory (there is no default location)."""
    cand = arg or os.environ.get("SLMT_REFERENCE_TREE")
    if cand and Path(cand).is_dir():
        return Path(cand)
    return None


def build_ref(ref_root=None, force: bool = False):
    """Build (or reuse) the reference extension; returns its path or None
    (None also when no reference tree is given and none was built before)."""
    so = built_path()
    if so is not None and not force:
        return so
    root = reference_tree(ref_root)
    if root is None:
        return None
    src = root / "kernels" / "kv_dequant_cuda.cu"
    if not src.exists():
        return None
    from torch.utils.cpp_extension import load
    REF_DIR.mkdir(exist_ok=True)
    load(name=EXT_NAME, sources=[str(src)], extra_include_paths=[str(src.parent)],
         extra_cuda_cflags=["-O3", "--expt-relaxed-constexpr", "-gencode=arch=compute_100a,code=sm_100a"],
         build_directory=str(REF_DIR), verbose=False)
    return built_path()


def load_ref():
    """Import the prebuilt reference extension (None if it was not built)."""
    so = built_path()
    if so is None:
        return None
    import torch  # noqa: F401  (the extension links against torch)
    loader = importlib.machinery.ExtensionFileLoader(EXT_NAME, str(so))
    spec = importlib.util.spec_from_file_location(EXT_NAME, str(so), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    print(build_ref(args[0] if args else None, force="--force" in sys.argv))
