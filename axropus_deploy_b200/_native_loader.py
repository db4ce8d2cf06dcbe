"""Loads the host-native extension ``_native`` (C++ AMF store, shard directory,
controllers). It is built in place by ``setup.py build_ext --inplace``; when it is
missing this module builds it (host C++ only, no CUDA) before importing, so a fresh
checkout works on a CPU-only machine."""
from __future__ import annotations

import importlib
import os
import subprocess
import sys
import threading

_LOCK = threading.Lock()
_MOD = None
_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_native(quiet: bool = True) -> None:
    env = dict(os.environ, AXR_SKIP_CUDA="1")
    cmd = [sys.executable, "setup.py", "build_ext", "--inplace"]
    out = subprocess.run(cmd, cwd=_ROOT, env=env, capture_output=quiet, text=True)
    if out.returncode != 0:
        raise RuntimeError("building the _native extension failed:\n" + (out.stderr or "")[-4000:])


def native():
    """Return the ``_native`` module, building it on first use if needed."""
    global _MOD
    if _MOD is not None:
        return _MOD
    with _LOCK:
        if _MOD is None:
            try:
                _MOD = importlib.import_module("axropus_deploy_b200._native")
            except ImportError:
                build_native()
                importlib.invalidate_caches()
                _MOD = importlib.import_module("axropus_deploy_b200._native")
    return _MOD
