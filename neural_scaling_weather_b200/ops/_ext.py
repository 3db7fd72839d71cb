"""Loader for the compiled sm_100a extension (``neural_scaling_weather_b200._C``).

The extension is built in-tree by ``setup.py build_ext --inplace`` (see
``__graft_entry__.build``).  CPU tensors never touch it.  On a CUDA device the fused
operators require it: :func:`require` raises instead of silently running a slower
PyTorch path, so a missing build cannot masquerade as a working one.
"""

from __future__ import annotations

import importlib
import os

_ext = None
_err = None


def load():
    global _ext, _err
    if _ext is not None or _err is not None:
        return _ext
    try:
        _ext = importlib.import_module("neural_scaling_weather_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _err = e
    return _ext


def available() -> bool:
    return load() is not None


def require():
    ext = load()
    if ext is None:
        raise RuntimeError(
            "neural_scaling_weather_b200._C is not built; run "
            "`python setup.py build_ext --inplace` (or __graft_entry__.build()) "
            f"before using CUDA tensors. Import error: {_err!r}"
        )
    return ext


def so_path() -> str | None:
    ext = load()
    return getattr(ext, "__file__", None) if ext is not None else None


ERROR_NAMES = {1: "bounded wait timed out", 2: "index out of bounds", 3: "invalid kernel argument"}


class DeviceError(RuntimeError):
    """A kernel of the extension recorded an error in the device error word: a bounded wait
    that ran out (its outputs are incomplete) or a rejected argument."""

    def __init__(self, code: int):
        self.code = int(code)
        super().__init__(f"device error word set: code {self.code} ({ERROR_NAMES.get(self.code, 'unknown')}); "
                         "the outputs of the kernels since the last check are not valid")


def check_device_errors() -> None:
    """Raise :class:`DeviceError` if a kernel recorded a bounded-wait timeout or a bounds
    violation (a synchronous read of the device error word, which is then cleared)."""
    ext = load()
    if ext is None:
        return
    code = ext.read_error_flag(True)
    if code != 0:
        raise DeviceError(code)


if os.environ.get("NSW_REQUIRE_EXT") == "1":  # pragma: no cover
    require()
