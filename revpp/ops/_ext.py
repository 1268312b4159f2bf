"""Loader for the compiled sm_100a extension (``revpp._C``).

CUDA tensors always go through the extension; when it is missing on a GPU
machine every op raises instead of silently falling back to PyTorch.
"""
from __future__ import annotations

import torch  # noqa: F401  (loads libc10 / libtorch before the extension)

_C = None
_ERR: Exception | None = None

try:  # pragma: no cover - depends on the build
    from revpp import _C as _C  # type: ignore[no-redef]
except Exception as e:  # noqa: BLE001
    _ERR = e


def ext():
    """Return the extension module or raise a clear error."""
    if _C is None:
        raise RuntimeError(
            "revpp CUDA extension is not built (python setup.py build_ext --inplace): "
            f"{_ERR!r}"
        )
    return _C


def available() -> bool:
    return _C is not None


def check_status(clear: bool = True) -> int:
    """Read the device error word written by bounded waits inside kernels."""
    c = ext()
    return c.status_read_and_clear() if clear else c.status_peek()
