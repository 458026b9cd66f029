"""Loader for the in-tree native modules.

``_C``  sm_100a CUDA kernels (built by ``python setup.py build_ext --inplace``).
``_rt`` host C++ runtime (block manager, IPC framing, GGUF index).

On a CUDA device every op goes through ``_C``; if the extension is missing the
op raises instead of falling back to PyTorch, so a GPU run can never pass on a
silent eager path.
"""
from __future__ import annotations

import importlib

import torch  # noqa: F401  (loads libc10 / libtorch that both extensions link against)

_C = None
_rt = None
_C_err: Exception | None = None
_rt_err: Exception | None = None

try:
    _C = importlib.import_module("openmini_v1_b200._C")
except Exception as e:  # pragma: no cover - depends on the build
    _C_err = e
try:
    _rt = importlib.import_module("openmini_v1_b200._rt")
except Exception as e:  # pragma: no cover
    _rt_err = e


def C():
    if _C is None:
        raise RuntimeError(
            "openmini_v1_b200._C (sm_100a kernels) is not built; run "
            f"`python setup.py build_ext --inplace` ({_C_err!r})")
    return _C


def rt():
    if _rt is None:
        raise RuntimeError(
            "openmini_v1_b200._rt (C++ runtime) is not built; run "
            f"`python setup.py build_ext --inplace` ({_rt_err!r})")
    return _rt


def have_C() -> bool:
    return _C is not None
