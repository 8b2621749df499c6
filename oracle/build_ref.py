"""Build recipe for the reference's own CUDA kernels (TEST / BASELINE
INFRASTRUCTURE ONLY -- the product never loads them).

Compiles the five source files of the reference's PyTorch extension
(warpgbm/cuda/{histogram_kernel,best_split_kernel,binner,predict}.cu and
node_kernel.cpp of quantverse/warpgbm v2.2.0) exactly where they lie in the
read-only reference checkout, for sm_100a, into ``oracle/_ref/`` (git-ignored;
the built module travels to the GPU box with the tree).  The reference's own
build system is not used: torch.utils.cpp_extension compiles the same five
files directly.

    python -m oracle.build_ref /path/to/reference   # build (or set WGB_REFERENCE)
    from oracle.build_ref import load                # import the built module (no sources needed)
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "wgb_ref_node_kernel"
SOURCES = ["histogram_kernel.cu", "best_split_kernel.cu", "binner.cu", "predict.cu", "node_kernel.cpp"]


def built_path():
    hits = sorted(glob.glob(os.path.join(OUT, NAME + "*.so")))
    return hits[0] if hits else None


def build(ref_root=None, force: bool = False):
    """Compile the reference extension of the checkout at ref_root (or
    $WGB_REFERENCE) into oracle/_ref/; returns the .so path.  Without a
    checkout (the GPU box) the prebuilt module is returned, or None."""
    ref_root = ref_root or os.environ.get("WGB_REFERENCE")
    src_dir = os.path.join(ref_root, "warpgbm", "cuda") if ref_root else None
    if not src_dir or not os.path.isdir(src_dir):
        return built_path()
    srcs = [os.path.join(src_dir, s) for s in SOURCES]
    so = built_path()
    if so and not force and all(os.path.getmtime(so) >= os.path.getmtime(s) for s in srcs):
        return so
    os.makedirs(OUT, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils.cpp_extension import load as cpp_load
    cpp_load(name=NAME, sources=srcs, build_directory=OUT, extra_cuda_cflags=["-O3"],
             extra_cflags=["-O3"], verbose=False)
    return built_path()


def load():
    """Import the built reference extension from oracle/_ref/ (raises if it
    was not built)."""
    so = built_path()
    if so is None:
        raise RuntimeError("reference CUDA extension not built (run python -m oracle.build_ref "
                           "where the reference checkout exists)")
    import torch  # noqa: F401  (the extension links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader(NAME, so)
    spec = importlib.util.spec_from_loader(NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    import sys
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, force=True))
