"""Builds the sm_100a extension in-tree (``eagle4_b200/_build/_e4.so``) and loads it.

The extension is compiled for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``): its kernels use
tcgen05/TMEM and TMA, which exist on no other target. The built library sits inside the package so it travels with
the source tree to the GPU machine; loading it never recompiles when the library is already present.
"""

from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys
from typing import Optional

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
NAME = "_e4"

SOURCES = ["bindings.cpp", "gemm.cu", "kernels.cu", "attention.cu", "recurrent.cu", "tree.cu", "comm.cu", "sampled.cu"]

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


def _so_path() -> Optional[str]:
    hits = sorted(glob.glob(os.path.join(BUILD, f"{NAME}*.so")))
    return hits[0] if hits else None


def build(verbose: bool = False):
    """Compile (or reuse) the extension and return the loaded module."""
    from torch.utils import cpp_extension

    os.makedirs(BUILD, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 1)))
    return cpp_extension.load(
        name=NAME,
        sources=[os.path.join(CSRC, s) for s in SOURCES],
        build_directory=BUILD,
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=CUDA_FLAGS,
        extra_ldflags=["-lcuda"],
        verbose=verbose,
    )


def load():
    """The extension module: the in-tree library if present, else a fresh build."""
    if NAME in sys.modules:
        return sys.modules[NAME]
    path = _so_path()
    if path is None:
        return build()
    import torch  # noqa: F401  (the extension links against torch's libraries)

    loader = importlib.machinery.ExtensionFileLoader(NAME, path)
    spec = importlib.util.spec_from_file_location(NAME, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[NAME] = mod
    return mod
