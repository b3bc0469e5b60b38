"""Build and load the in-tree sm_100a extension ``d3d_b200_C``.

The shared object is built into ``d3d_b200/ops/_build/`` (in the source tree,
so it travels with the repository snapshot to the GPU machine) with
``-gencode arch=compute_100a,code=sm_100a``.  :func:`load` imports the built
``.so`` directly and only invokes the compiler when it is missing, or when
``D3D_REBUILD=1``.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
# D3D_DEBUG=1 selects a separate debug build (device bounds checks on the
# indices the kernels take from step inputs: KV slots, pages, token ids)
DEBUG = os.environ.get("D3D_DEBUG") == "1"
BUILD_DIR = HERE / ("_build_debug" if DEBUG else "_build")
NAME = "d3d_b200_C_debug" if DEBUG else "d3d_b200_C"

SOURCES = ["bindings.cpp", "gemm_tcgen05.cu", "fused.cu", "attention.cu", "attention_tc.cu", "handoff.cu",
           "train_kernels.cu", "tp.cu", "fsdp.cu"]

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]

_mod = None


def so_path() -> Path:
    return BUILD_DIR / f"{NAME}.so"


def build(verbose: bool = False):
    """Compile the extension for sm_100a (works without a GPU)."""
    import torch  # noqa: F401  (needed before cpp_extension)
    from torch.utils import cpp_extension

    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    srcs = [str(CSRC / s) for s in SOURCES if (CSRC / s).exists()]
    mod = cpp_extension.load(
        name=NAME,
        sources=srcs,
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=CUDA_FLAGS + (["-DD3D_DEBUG_BOUNDS"] if DEBUG else []),
        extra_include_paths=[str(CSRC)],
        build_directory=str(BUILD_DIR),
        verbose=verbose,
        with_cuda=True,
    )
    return mod


def stale_sources() -> list:
    """Kernel sources changed after the shared object was built."""
    path = so_path()
    if not path.exists():
        return []
    t = path.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh"))
    return [p.name for p in deps if p.exists() and p.stat().st_mtime > t + 1.0]


def load():
    """Import the built extension (building it first if absent).  A shared
    object older than its sources is rebuilt when a compiler is at hand
    (``D3D_REBUILD=1`` forces it) and refused otherwise, so a stale binary
    never runs against newer Python code."""
    global _mod
    if _mod is not None:
        return _mod
    import torch  # noqa: F401

    path = so_path()
    stale = stale_sources()
    if os.environ.get("D3D_REBUILD") == "1" or not path.exists() or stale:
        _mod = build()
        return _mod
    loader = importlib.machinery.ExtensionFileLoader(NAME, str(path))
    spec = importlib.util.spec_from_file_location(NAME, str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[NAME] = mod
    _mod = mod
    return mod


def build_debug():
    """Compile the debug build (bounds-checked kernels) into ``_build_debug``
    in a child process (the build variant is chosen at import time)."""
    import subprocess
    env = dict(os.environ, D3D_DEBUG="1")
    subprocess.run([sys.executable, "-c", "from d3d_b200.ops import build; build.build()"], env=env,
                   check=True, cwd=str(HERE.parents[1]))


def load_debug():
    """The debug build (bounds-checked kernels), built on first use (or when
    older than its sources) into ``_build_debug`` whatever ``D3D_DEBUG``
    says; returns the module."""
    path = HERE / "_build_debug" / "d3d_b200_C_debug.so"
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh"))
    if not path.exists() or any(p.exists() and p.stat().st_mtime > path.stat().st_mtime + 1.0 for p in deps):
        build_debug()
    name = "d3d_b200_C_debug"
    loader = importlib.machinery.ExtensionFileLoader(name, str(path))
    spec = importlib.util.spec_from_file_location(name, str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod
