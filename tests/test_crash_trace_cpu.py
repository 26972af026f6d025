"""The extension's opt-in native crash backtrace: a child process that loads the
extension with ``AVGEN_NATIVE_BACKTRACE=1`` and then dereferences a null
pointer on the host prints the native frames, then Python's fault handler
prints the Python stack, and the child dies of the signal (host only: the
fault is a CPU segmentation fault in a throwaway process, no GPU involved)."""
from __future__ import annotations

import os
import signal
import subprocess
import sys

import pytest

CHILD = """
import ctypes, faulthandler
faulthandler.enable()
from avgen_b200.ops._ext import load
load()
ctypes.string_at(0)
"""


def test_native_backtrace_then_python_stack() -> None:
    try:
        from avgen_b200.ops._ext import load

        load()
    except RuntimeError:
        pytest.skip("extension not built")
    env = dict(os.environ, AVGEN_NATIVE_BACKTRACE="1")
    proc = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=300,
                          cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert proc.returncode == -signal.SIGSEGV, (proc.returncode, proc.stderr[-2000:])
    err = proc.stderr
    assert "native backtrace" in err
    assert "Fatal Python error" in err and "string_at" in err  # the previous handler still ran


def test_install_is_idempotent() -> None:
    try:
        from avgen_b200.ops._ext import load

        ext = load()
    except RuntimeError:
        pytest.skip("extension not built")
    code = "from avgen_b200.ops._ext import load; e = load(); print(e.install_crash_backtrace(), e.install_crash_backtrace())"
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                         cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert out.stdout.split() == ["True", "False"], out.stderr[-2000:]
    assert hasattr(ext, "install_crash_backtrace")
