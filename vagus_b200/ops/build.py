"""Build and load the in-tree sm_100a extension (``vagus_b200_C``).

The extension is compiled with ``torch.utils.cpp_extension`` into
``vagus_b200/ops/_build`` (in-tree, so a copied checkout carries the built
``.so``) with ``-gencode arch=compute_100a,code=sm_100a`` in the nvcc flags,
which also keeps torch from adding its own architecture list.  A SHA-256 of
the sources and flags is stored beside the library; ``load()`` imports the
existing library directly when the hash matches and rebuilds otherwise.
"""

from __future__ import annotations

import hashlib
import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

NAME = "vagus_b200_C"
HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
# VAGUS_BOUNDS_CHECK=1 selects the bounds-checked build (-DVAGUS_BOUNDS_CHECK:
# hand-computed global indices are checked against their tensors, a miss is
# recorded in the device error word and the access skipped), kept in its own
# directory beside the normal one.
BOUNDS_CHECK = os.environ.get("VAGUS_BOUNDS_CHECK", "") not in ("", "0")
BUILD_DIR = HERE / ("_build_bounds" if BOUNDS_CHECK else "_build")

SOURCES = [
    "bindings.cpp", "bind_seq.cpp", "bind_attn.cpp", "bind_comm.cpp",
    "gemm.cu", "norm.cu", "elementwise.cu", "conv.cu", "gdn_gates.cu", "gdr.cu", "gdr_intra.cu", "attention.cu",
    "comm.cu", "ce_noalloc.cu", "kda.cu", "kda_intra.cu", "mobius.cu",
]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-diag-suppress=177,550"]
CXX_FLAGS = ["-O3", "-std=c++17"]
if BOUNDS_CHECK:
    CUDA_FLAGS = CUDA_FLAGS + ["-DVAGUS_BOUNDS_CHECK=1"]


def _sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def source_hash() -> str:
    h = hashlib.sha256()
    for p in sorted(_sources()) + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(CUDA_FLAGS + CXX_FLAGS).encode())
    return h.hexdigest()


def _lib_path() -> Path:
    return BUILD_DIR / f"{NAME}.so"


def build(verbose: bool = False):
    """Compile every CUDA/C++ source for sm_100a and return the module."""
    from torch.utils.cpp_extension import load as cpp_load
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    mod = cpp_load(name=NAME, sources=[str(p) for p in _sources()], build_directory=str(BUILD_DIR),
                   extra_cflags=CXX_FLAGS, extra_cuda_cflags=CUDA_FLAGS, verbose=verbose,
                   with_cuda=True)
    (BUILD_DIR / "SOURCES_SHA256").write_text(source_hash())
    return mod


def load(allow_build: bool = True):
    """Import the built library (building it first if it is missing or stale)."""
    if NAME in sys.modules:
        return sys.modules[NAME]
    lib = _lib_path()
    stamp = BUILD_DIR / "SOURCES_SHA256"
    if lib.exists() and stamp.exists() and stamp.read_text().strip() == source_hash():
        import torch  # noqa: F401  (libtorch symbols must be loaded first)
        loader = importlib.machinery.ExtensionFileLoader(NAME, str(lib))
        spec = importlib.util.spec_from_file_location(NAME, str(lib), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        sys.modules[NAME] = mod
        return mod
    if not allow_build:
        raise RuntimeError(f"{NAME} is not built (run vagus_b200.ops.build.build())")
    mod = build()
    sys.modules[NAME] = mod
    return mod


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", _lib_path())
