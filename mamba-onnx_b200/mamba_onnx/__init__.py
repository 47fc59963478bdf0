"""Mamba selective-scan custom ops for ONNX Runtime — CUDA (sm_100a) backend.

Drop-in for the reference package's loader (acmiyaguchi/mamba-onnx
src/mamba_onnx/__init__.py): the same three functions with the same argument
meaning and errors, plus a ``cuda`` backend that resolves to
``libmamba_ops_cuda.so``. The library registers domain ``mamba`` with
SelectiveScan, SelectiveScanExact, SelectiveScanFused and
SelectiveScanFusedExact for the CUDAExecutionProvider::

    import onnxruntime as ort
    import mamba_onnx
    opts = ort.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    sess = ort.InferenceSession("model.onnx", opts, providers=["CUDAExecutionProvider"])

There is no CPU fallback: asking for ``cuda`` when the CUDA library is absent
raises FileNotFoundError.

``mamba_onnx.cuda.selective_scan`` runs the same kernels directly on torch
CUDA tensors through the library's C ABI (include/mamba_scan.h).
"""
import sys
from pathlib import Path

__version__ = "0.1.0"

_PKG_DIR = Path(__file__).parent
_BUILD_LIB_DIR = _PKG_DIR.parent / "build" / "lib"

# Search directories: build/lib/ first (dev), then the package dir (where the
# in-tree build writes libmamba_ops_cuda.so) — __init__.py:19-22 of the reference.
_SEARCH_DIRS = [_BUILD_LIB_DIR, _PKG_DIR]

_BACKEND_LIBS = {
    "cuda": "libmamba_ops_cuda.so",
    "zig": "libmamba_ops_zig.so",
    "cpp": "libmamba_ops_cpp.so",
}


def available_backends() -> list[str]:
    """List the backends whose library is present (cuda, and cpp/zig if installed)."""
    found = []
    seen = set()
    for search_dir in _SEARCH_DIRS:
        if not search_dir.is_dir():
            continue
        for path in sorted(search_dir.glob("libmamba_ops*.so")):
            if path.name in seen:
                continue
            seen.add(path.name)
            for backend, lib in _BACKEND_LIBS.items():
                if path.name == lib and backend not in found:
                    found.append(backend)
    return found


def get_library_path(backend: str = "auto") -> str:
    """Path to the shared library of a backend.

    Args:
        backend: "cuda", "cpp", "zig", or "auto" (cuda first, then zig, then cpp).

    Raises:
        FileNotFoundError: if no matching library is found.
        ValueError: on an unknown backend name.
    """
    if backend == "auto":
        candidates = [_BACKEND_LIBS["cuda"], _BACKEND_LIBS["zig"], _BACKEND_LIBS["cpp"]]
    elif backend in _BACKEND_LIBS:
        candidates = [_BACKEND_LIBS[backend]]
    else:
        raise ValueError(f"unknown backend {backend!r}; expected one of "
                         f"{sorted(_BACKEND_LIBS) + ['auto']}")
    if not sys.platform.startswith("linux"):
        raise FileNotFoundError("the cuda backend is built for Linux only")
    for search_dir in _SEARCH_DIRS:
        for name in candidates:
            path = search_dir / name
            if path.exists():
                return str(path)
    searched = ", ".join(str(d) for d in _SEARCH_DIRS)
    raise FileNotFoundError(
        f"No mamba_ops library found for backend {backend!r}. Searched: {searched}\n"
        f"Build with: python -c 'import __graft_entry__ as g; g.build()' (repository root)"
    )


def register_custom_ops(session_options, backend: str = "auto") -> str:
    """Register the Mamba custom ops with ONNX Runtime session options.

    Args:
        session_options: an onnxruntime.SessionOptions instance (anything with
            register_custom_ops_library(path)).
        backend: "cuda", "cpp", "zig", or "auto".

    Returns:
        Path of the library that was loaded.
    """
    lib_path = get_library_path(backend)
    session_options.register_custom_ops_library(lib_path)
    return lib_path


__all__ = [
    "register_custom_ops",
    "get_library_path",
    "available_backends",
    "__version__",
]
