"""Build and load the sm_100a CUDA extension (``tinytron_b200_C``).

The extension is compiled in-tree (``build/tt_ext/``) with
``-gencode arch=compute_100a,code=sm_100a`` only; nothing is JIT-compiled at
import time.  ``load()`` imports the prebuilt shared object and raises loudly if
it is missing, so a GPU run can never silently fall back to another code path.
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

REPO_ROOT = Path(__file__).resolve().parents[2]
CSRC = REPO_ROOT / "csrc"
BUILD_DIR = REPO_ROOT / "build" / "tt_ext"
EXT_NAME = "tinytron_b200_C"

SOURCES = [
    "bindings.cpp",
    "runtime/status.cu",
    "runtime/comm.cu",
    "runtime/ulysses.cu",
    "gemm/gemm.cu",
    "gemm/skinny.cu",
    "fused/norm.cu",
    "fused/elementwise.cu",
    "fused/sample.cu",
    "attn/attn_fwd.cu",
    "attn/attn_bwd.cu",
    "attn/decode.cu",
    "moe/moe.cu",
    "moe/ep.cu",
]

CUDA_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]

_module = None


def so_path() -> Path:
    return BUILD_DIR / f"{EXT_NAME}.so"


def build(verbose: bool = False, ptxas_verbose: bool = False):
    """Compile every CUDA source for sm_100a into ``build/tt_ext``."""
    from torch.utils import cpp_extension

    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    flags = list(CUDA_FLAGS)
    if ptxas_verbose:
        flags.append("-Xptxas=-v")
    mod = cpp_extension.load(
        name=EXT_NAME,
        sources=[str(CSRC / s) for s in SOURCES],
        build_directory=str(BUILD_DIR),
        extra_cuda_cflags=flags,
        extra_cflags=["-O3", "-std=c++17"],
        extra_include_paths=[str(CSRC)],
        verbose=verbose,
        is_python_module=True,
    )
    global _module
    _module = mod
    return mod


def load():
    """Import the prebuilt extension; raise if it has not been built."""
    global _module
    if _module is not None:
        return _module
    if EXT_NAME in sys.modules:
        _module = sys.modules[EXT_NAME]
        return _module
    path = so_path()
    if not path.exists():
        raise RuntimeError(
            f"tinytron_b200 CUDA extension not built ({path} missing); "
            "run `python -c 'import __graft_entry__ as g; g.build()'` first"
        )
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(EXT_NAME, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[EXT_NAME] = mod
    _module = mod
    return mod


def available() -> bool:
    try:
        load()
        return True
    except Exception:
        return False
