"""Loader of the compiled sm_100a kernels (``everserve_b200._C``).

The extension is built in-tree (``python setup.py build_ext --inplace``), or, on a node without
the build, fetched from another node's compile cache and named by ``ES_EXTENSION_PATH``. On a machine with a GPU a
missing or broken extension is an error: no op silently runs another implementation on a CUDA
tensor. CPU tensors use the PyTorch reference ops in :mod:`everserve_b200.ops.ref`, which are the
CPU engine's arithmetic and the kernels' numerical oracle.

Reference parity: the reference's loader builds its extension with
``torch.utils.cpp_extension.load`` and refuses a mismatched prebuilt stamp
(core/everserve/kernels.py:170-221); here the build is ahead-of-time and the import is the check.
"""

from __future__ import annotations

import importlib
import importlib.util
import os
import sys

_C = None
_ERR: Exception | None = None


def load():
    """Import the extension once; raise with the original error if it cannot be imported."""
    global _C, _ERR
    if _C is not None:
        return _C
    if _ERR is not None:
        raise RuntimeError(f"everserve_b200._C is not available: {_ERR}") from _ERR
    try:
        import torch  # noqa: F401 - the extension links against torch's libraries, loaded by this import

        path = os.environ.get("ES_EXTENSION_PATH", "")
        if path:  # a build fetched from another node's compile cache
            spec = importlib.util.spec_from_file_location("everserve_b200._C", path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            sys.modules["everserve_b200._C"] = mod
            _C = mod
        else:
            _C = importlib.import_module("everserve_b200._C")
    except Exception as e:  # noqa: BLE001 - re-raised with context below
        _ERR = e
        raise RuntimeError(
            "everserve_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"in {os.path.dirname(os.path.dirname(os.path.abspath(__file__)))}: {e}"
        ) from e
    return _C


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def so_path() -> str | None:
    """Path of the loaded extension file (for provenance in logs and bench output)."""
    return getattr(load(), "__file__", None) if available() else None
