"""Loader of the sm_100a kernel extension ``_C``.

CUDA tensors always run through the extension; if it is missing on a machine with a
GPU the call raises instead of silently falling back to PyTorch, so a GPU run can
never pass on a fallback path. CPU tensors use the plain PyTorch oracles next to
each op (the references the kernel tests compare against)."""
from __future__ import annotations

import importlib
import os

_C = None
_ERR = None
# Kernels of this framework launched so far (per process). Each wrapper call adds the
# number of kernels it launches; CUDA-graph replays add what their capture recorded.
LAUNCHES = [0]
_KERNELS_PER_CALL = {
    # split kernel + combine (split-KV or shared-prefix merge)
    "decode_attention": lambda a: 2 if (a[14] > 1 or (len(a) > 19 and a[19] is not None)) else 1,
    # attention kernel + combine unless the partials are kept for a later merge
    "prefill_attention_tc": lambda a: 2 if (a[14] > 1 and not (len(a) > 20 and a[20])) else 1,
    "prefill_attention": lambda a: 2 if a[17] > 1 else 1,
    # amax (+ scales) + encode; NVFP4 is one kernel
    "codec_encode": lambda a: 1 if a[1] == 3 else 3,
}


class _Counted:
    def __init__(self, mod):
        self._mod = mod
        self.__file__ = mod.__file__

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn) or name in ("decode_num_splits", "dense_stream_nt", "dense_stream_splits",
                                                   "dense_stream_workspace"):
            return fn
        per = _KERNELS_PER_CALL.get(name)

        def call(*a):
            LAUNCHES[0] += per(a) if per else 1
            return fn(*a)

        return call


def launches() -> int:
    return LAUNCHES[0]


def cuda_ext():
    global _C, _ERR
    if _C is not None:
        return _C
    try:
        _C = _Counted(importlib.import_module("axropus_deploy_b200._C"))
    except ImportError as e:  # pragma: no cover - exercised on GPU boxes only
        _ERR = e
        raise RuntimeError(
            "axropus_deploy_b200._C (the sm_100a kernels) is not built; run "
            "`python setup.py build_ext --inplace` (or __graft_entry__.build()). "
            f"Import error: {e}") from e
    return _C


def ext_path() -> str:
    return os.path.abspath(cuda_ext().__file__)
