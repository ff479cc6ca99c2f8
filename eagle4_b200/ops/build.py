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

SOURCES = ["bindings.cpp", "gemm.cu", "kernels.cu", "attention.cu", "recurrent.cu", "tree.cu", "comm.cu", "sampled.cu",
           "moe.cu"]

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


HASH_FILE = os.path.join(BUILD, f"{NAME}.srchash")


def _so_path() -> Optional[str]:
    hits = sorted(glob.glob(os.path.join(BUILD, f"{NAME}*.so")))
    return hits[0] if hits else None


def source_hash() -> str:
    """SHA-256 over every source and header of the extension and the compiler flags: the identity of a build."""
    import hashlib

    h = hashlib.sha256()
    files = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp"))
                   + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")))
    for f in files:
        h.update(os.path.basename(f).encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(CUDA_FLAGS).encode())
    return h.hexdigest()


def _built_hash() -> Optional[str]:
    try:
        with open(HASH_FILE) as f:
            return f.read().strip()
    except OSError:
        return None


def build(verbose: bool = False):
    """Compile (or reuse) the extension and return the loaded module."""
    from torch.utils import cpp_extension

    os.makedirs(BUILD, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 1)))
    digest = source_hash()
    mod = cpp_extension.load(
        name=NAME,
        sources=[os.path.join(CSRC, s) for s in SOURCES],
        build_directory=BUILD,
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=CUDA_FLAGS,
        extra_ldflags=["-lcuda"],
        verbose=verbose,
    )
    with open(HASH_FILE + ".tmp", "w") as f:
        f.write(digest)
    os.replace(HASH_FILE + ".tmp", HASH_FILE)
    return mod


def load():
    """The extension module: the in-tree library if it was built from the current sources, else a fresh build.

    A library whose recorded source hash differs from the sources beside it (a stale build shipped with newer
    sources) is rebuilt, never run."""
    if NAME in sys.modules:
        return sys.modules[NAME]
    path = _so_path()
    if path is None or _built_hash() != source_hash():
        return build()
    import torch  # noqa: F401  (the extension links against torch's libraries)

    loader = importlib.machinery.ExtensionFileLoader(NAME, path)
    spec = importlib.util.spec_from_file_location(NAME, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[NAME] = mod
    return mod
