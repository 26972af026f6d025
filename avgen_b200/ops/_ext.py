"""Loader for the sm_100a CUDA extension ``avgen_b200._C``.

The extension is built in-tree (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``). On a machine with a CUDA device, a missing or
unloadable extension is an error: every GPU op of this package runs a
hand-written kernel and there is no silent PyTorch fallback.
"""
from __future__ import annotations

import importlib
import os
from types import ModuleType

import torch

_EXT: ModuleType | None = None
_ERR: BaseException | None = None


def load() -> ModuleType:
    """Return the compiled extension, importing it on first use.

    Raises:
        RuntimeError: If the extension cannot be imported.
    """
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    try:
        _EXT = importlib.import_module("avgen_b200._C")
    except BaseException as exc:  # noqa: BLE001 - re-raised with context below
        _ERR = exc
        raise RuntimeError(
            "avgen_b200._C (the sm_100a kernels) is not built or failed to load; "
            "run `python setup.py build_ext --inplace` in the repository root"
        ) from exc
    if os.environ.get("AVGEN_NATIVE_BACKTRACE", "0") == "1":
        _EXT.install_crash_backtrace()  # native frames on a host crash, then Python's fault handler
    return _EXT


def available() -> bool:
    """Whether the extension imports (it may still need a B200 to run)."""
    try:
        load()
        return True
    except RuntimeError:
        return False


def is_sm100(device: torch.device | int | None = None) -> bool:
    """Whether ``device`` is a compute-capability 10.x GPU (B200 family)."""
    if not torch.cuda.is_available():
        return False
    major, _ = torch.cuda.get_device_capability(device)
    return major == 10


def check_errors(device: torch.device | int | None = None, *, clear: bool = True) -> int:
    """Read the device error word that bounded in-kernel waits write into.

    Returns:
        0 when no kernel timed out; otherwise the first error code recorded.
    """
    ext = load()
    index = torch.cuda.current_device() if device is None else torch.device("cuda", device).index if isinstance(device, int) else device.index
    code = int(ext.read_error(int(index)))
    if code and clear:
        ext.clear_error(int(index))
    return code
